// Rasterisation of closed fills and open strokes, forward and backward
// (sm_100a).
//
// The unit of work is a strip: 4 pixel rows x 16 columns of a 16x16 tile, one
// warp, two horizontally adjacent pixels per lane.  The kernels are
// persistent: every warp takes its first strip by its global warp id and the
// next ones from a device counter, in the heaviest-first order computed by
// the staging pass, so the SMs stay evenly loaded to the end of the launch.
// A strip's geometry was staged once per frame (stage.cuh): the compact list
// of the edges that come within d_thr of the strip, per intersect, plus
// per-row winding offsets for far edges right of the tile.  Each warp brings
// its strip's list into its own shared-memory buffers with cp.async.bulk
// copies of up to kWChunk records, double-buffered and completed on the
// warp's own mbarriers, and walks the intersects on its own: there is no CTA
// barrier until the launch ends.
//
// Why visiting only near edges is exact: d_thr is the distance beyond which a
// pixel's coverage is saturated for the primitive (fill: exactly 1.0f inside
// and below alpha_min outside; stroke: below alpha_min).  A pixel closer than
// d_thr to the polyline has its closest edge in its strip's list, so its
// minimum distance is the exact one; a farther pixel gets a saturated
// coverage from whatever edges it sees, identical to visiting every edge.
// The crossing test needs all edges that span the pixel's row and lie right
// of it: near ones are tested per pixel, far ones are the per-row offsets.
// This is the reference's per-pixel loop over every edge of every intersect
// (manbo/ops/cubic_splatting.py:1070-1136 forward, :1429-1501 backward;
// cubic_polyline_splatting.py:175-216, :480-529) with the same formulas in
// the same order and exp = cs_expf.
//
// The backward walks the intersects in reverse from the warp's largest
// final_idx with T <- T / (1 - alpha), takes the first-minimum closest edge
// (the reference's strict-< rule in edge order), reduces per-primitive
// gradients over the warp (four values per shuffle butterfly) before one
// atomic per primitive value, and accumulates edge gradients per staged record
// in shared memory before one global atomic per edge and chunk (each warp
// first sums its lanes' contributions per distinct closest edge).  With visit
// lists it walks only the intersects that composited a pixel of the strip;
// with a fill forward's winner codes it evaluates only each pixel's closest
// record of such an intersect (and whether the pixel is inside) instead of
// every record.  Its per-pixel coverage, reciprocals and square root use the
// fast hardware forms: the forward image must match the oracle bit for bit,
// the gradients only within the reference's tolerance.
#include "stage.cuh"

namespace cs {

constexpr int kRW = 4;                // warps per CTA (independent strip processors)
constexpr int kRT = 32 * kRW;
constexpr int kWChunk = 64;           // staged records per warp buffer
constexpr int kAcc = 10;              // per-intersect gradient accumulators
constexpr int kSpinLimit = 1 << 22;   // mbarrier polls before reporting a timeout

struct RasterArgs {
  const int* pids;
  const int* bins;
  const int2* dlr;       // per tile: first staged record, per-strip capacity
  const IMeta* meta;
  const int2* istrip;    // per intersect and strip: (first record, record count)
  const int* rowoff;     // [I][16] packed row winding offsets (fill)
  const DEntry* dl;
  const int* order;      // optional unit lists (stage.cuh), heaviest bucket first
  int* order_next;       // forward: optional unit lists for the backward, by measured work
  int* visits;           // optional per-strip lists of the intersects that composited a pixel
                         // of the strip: the forward writes them, the backward walks them
  unsigned short* winners;  // optional, beside the visit lists: per listed visit and lane, the
                            // two pixels' closest-record codes (see winner_code)
  const float* bg;
  int H, W, tbx, r0, nunits;
  int vec2;              // W even and per-pixel buffers 8-byte aligned: a lane's two
                         // pixels move as one 8-byte access per plane
  int* status;
  unsigned* queue;       // workspace: next dynamically taken unit
  unsigned* ticket;      // workspace: CTA completion ticket
  float* partials;       // workspace: per-unit sums of squared differences
  // forward outputs
  float* out;
  float* fts;
  int* fidx;
  float* out_chw;
  const float* loss_tgt;     // optional [3, H, W] target: fused SSE / MSE
  float* loss_out;           // [2]: sse of the band, sse / (3 H W)
  // backward
  const float* fts_in;
  const int* fidx_in;
  const float* v_out;
  const float* out_img;
  const float* tgt;
  const float* mse_scale;
  float* v_edges;
  float* v_colors;
  float* v_opac;
  float* v_inv;
  float* v_sw;
  float* contrib;
  float* icontrib;
};

// Tile, strip and first record of a unit (unit = kStrips * band tile + strip).
struct UnitGeom {
  long long tile;
  int tx, ty, st, rs, re;
  long long base;  // first record of the strip's list
};

// A strip's visit list: count, then up to re - rs intersect ids in ascending
// order.  Tile t's four lists start at 4 (rs + t), so the lists of all tiles
// with intersects fit 4 (I + num_tiles) ints without overlap (tiles without
// intersects have no list).
__device__ __forceinline__ long long visit_base(const UnitGeom& g) {
  return 4LL * ((long long)g.rs + g.tile) + (long long)g.st * (g.re - g.rs + 1);
}

__device__ __forceinline__ UnitGeom unit_geom(const RasterArgs& A, int unit) {
  UnitGeom g;
  const int trel = unit / kStrips;
  g.st = unit - trel * kStrips;
  const int ry = trel / A.tbx;
  g.tx = trel - ry * A.tbx;
  g.ty = A.r0 + ry;
  g.tile = (long long)g.ty * A.tbx + g.tx;
  g.rs = __ldg(A.bins + 2 * g.tile);
  g.re = __ldg(A.bins + 2 * g.tile + 1);
  const int2 dl = A.dlr[g.tile];  // loaded beside the ranges (every tile has an entry)
  g.base = g.re > g.rs ? (long long)dl.x + (long long)g.st * dl.y : 0;
  return g;
}

// Number of records of intersects [rs, k] in strip st's list.
__device__ __forceinline__ int strip_records_upto(const RasterArgs& A, int k, int st) {
  const int2 r = A.istrip[(long long)k * kStrips + st];
  return r.x + r.y;
}

// Next unit of this warp: the first by warp id, the rest from the counter.
__device__ __forceinline__ int next_unit(const RasterArgs& A) {
  unsigned v = 0u;
  if ((threadIdx.x & 31) == 0) v = gridDim.x * kRW + atomicAdd(A.queue, 1u);
  return (int)__shfl_sync(0xffffffffu, v, 0);
}

// The last CTA to finish resets the counters (and reduces the loss partials
// in a fixed order when asked), so the workspace is ready for the next launch.
__device__ __forceinline__ void finish_launch(const RasterArgs& A, bool reduce_loss) {
  __shared__ bool last;
  __shared__ float red[kRW];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(A.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (reduce_loss) {
    float v = 0.0f;
    for (int q = threadIdx.x; q < A.nunits; q += kRT) v += A.partials[q];
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < kRW; ++w) t += red[w];
      A.loss_out[0] = t;
      A.loss_out[1] = t / (3.0f * (float)A.H * (float)A.W);
    }
  }
  if (threadIdx.x == 0) {
    *A.queue = 0u;
    *A.ticket = 0u;
  }
}

// Per-warp batch of up to 32 consecutive intersects' records in shared
// memory: the IMeta record (three 16-byte parts), the strip's record range and
// the strip's four packed row offsets.  One coalesced load per lane replaces a
// chain of dependent global loads per intersect.
struct IBatch {
  int4 m[3][32];
  int2 rg[32];
  int4 ro[32];
  int kk[32];  // the intersect ids (-1: a listed id outside the tile, skipped)
};

// Whether intersect (meta m0..m2, strip range rg, row offsets ro) can change
// any pixel of the strip.  With no near edge every pixel is farther than d_thr
// from the polyline, so its coverage is saturated: a stroke's op * cov is below
// alpha_min, and so is a fill's in every row the far-edge offsets put outside.
// Such an intersect composites nothing in the forward and gets no gradient in
// the backward, exactly as in the per-pixel loop.  The guard keeps the
// pathological primitives (no edges, infinite or huge width, opacity or
// d_thr) on the full path, where op * cov need not stay below alpha_min.
template <bool STROKE>
__device__ __forceinline__ bool intersect_active(const int4& m0, const int4& m1, const int4& m2,
                                                 const int2& rg, const int4& ro) {
  if (rg.y > 0) return true;
  const float op = __int_as_float(m1.w), dthr = __int_as_float(m2.z);
  if (!(op <= 1e20f && dthr <= 1e6f)) return true;
  if (STROKE) return false;
  const int r[4] = {ro.x, ro.y, ro.z, ro.w};
  bool inside = false;
#pragma unroll
  for (int q = 0; q < kStripRows; ++q)
    inside |= (m0.w == 0) ? (row_cnt(r[q]) & 1) != 0 : row_wind(r[q]) != 0;
  return inside;
}

// Loads n intersects into the warp's batch -- k0 .. k0 + n - 1, or the ids
// lst[0 .. n) of a visit list, each checked against the tile's [rs, re) -- and
// returns the mask of those that can change a pixel of the strip (bit j:
// batch entry j).
template <bool STROKE>
__device__ __forceinline__ unsigned load_batch(const RasterArgs& A, const int* lst, int k0, int n,
                                               int st, int rs, int re, IBatch& b,
                                               bool have_id = false, int lane_id = 0) {
  const int lane = threadIdx.x & 31;
  bool act = false;
  __syncwarp();  // every lane is done with the previous batch
  if (lane < n) {
    int kid = k0 + lane;
    if (lst) {
      kid = have_id ? lane_id : __ldg(lst + lane);  // lane_id: lst[lane], loaded by the caller
      if (kid < rs || kid >= re) {  // not a list the forward wrote for this strip
        if (A.status) atomicExch(A.status, CS_ERR_ARG);
        kid = -1;
      }
    }
    b.kk[lane] = kid;
  }
  if (lane < n && b.kk[lane] >= 0) {
    const long long k = b.kk[lane];
    const int4* q = reinterpret_cast<const int4*>(A.meta + k);
    const int4 m0 = __ldg(q), m1 = __ldg(q + 1), m2 = __ldg(q + 2);
    const int2 rg = __ldg(A.istrip + k * kStrips + st);
    int4 ro = make_int4(0, 0, 0, 0);
    if (!STROKE) ro = __ldg(reinterpret_cast<const int4*>(A.rowoff + k * 16 + st * kStripRows));
    b.m[0][lane] = m0;
    b.m[1][lane] = m1;
    b.m[2][lane] = m2;
    b.rg[lane] = rg;
    b.ro[lane] = ro;
    act = intersect_active<STROKE>(m0, m1, m2, rg, ro);
  }
  __syncwarp();
  return __ballot_sync(0xffffffffu, act);
}

__device__ __forceinline__ void batch_meta(const IBatch& b, int j, IMeta& m) {
  const int4 x = b.m[0][j], y = b.m[1][j], z = b.m[2][j];
  m.dstart = x.x; m.dcount = x.y; m.pid = x.z; m.rule = x.w;
  m.c0 = __int_as_float(y.x); m.c1 = __int_as_float(y.y);
  m.c2 = __int_as_float(y.z); m.op = __int_as_float(y.w);
  m.a = __int_as_float(z.x); m.b = __int_as_float(z.y); m.dthr = __int_as_float(z.z);
  m.spare = 0.0f;
}

// Packed row offset of this lane's pixel row (row lane / 8 of the strip).
__device__ __forceinline__ int batch_rowoff(const IBatch& b, int j) {
  return reinterpret_cast<const int*>(&b.ro[j])[(threadIdx.x & 31) >> 3];
}

// ---------------------------------------------------------------------------
// bulk copies into shared memory (non-multicast cp.async.bulk + mbarrier)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Issued by one thread: arrive on `bar` expecting `bytes`, then copy.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait of one warp on its own buffer's mbarrier; the outcome is agreed
// by the warp.  On timeout the device status is set and the warp stops.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status) {
  bool ok = false;
  for (int i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) {
      ok = true;
      break;
    }
  }
  const bool all = __all_sync(0xffffffffu, ok);
  if (!all && (threadIdx.x & 31) == 0 && status) atomicExch(status, CS_ERR_TIMEOUT);
  return all;
}

// Wait for the next completion of buffer b's barrier (b = 0 or 1; bit b of
// phase holds its parity and flips with every completion).
__device__ __forceinline__ bool wait_buffer(uint64_t* bars, int b, uint32_t& phase, int* status) {
  const bool ok = warp_wait(&bars[b], (phase >> b) & 1u, status);
  phase ^= 1u << b;
  return ok;
}

// 16-byte copies global -> shared that complete asynchronously (cp.async,
// non-bulk): each thread's copies are grouped by cp_async_commit and waited
// for by that thread with cp_async_wait_all.  The .ca form keeps the line in
// L1 (lanes of a strip often share a winning record), .cg reads through L2.
__device__ __forceinline__ void cp_async16_ca(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async16_cg(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------------------
// per-pixel arithmetic (reference formulas, written order)

// Squared distance to the edge of record (A, B): proj = (w . v) / |v|^2
// clamped to [0, 1], closest point c = p0 + proj v, d2 = |c - p|^2, with one
// fused multiply-add each for the dot product, the closest point and the
// squared length (the CPU oracle evaluates the same expressions).
__device__ __forceinline__ float seg_d2(float px, float py, float wy, const float4& A,
                                        const float4& B, float& proj, float& cx, float& cy) {
  const float wx = px - A.x;
  float pr = __fmaf_rn(wx, A.z, wy * A.w) * B.x;
  pr = fmaxf(0.0f, fminf(1.0f, pr));
  cx = __fmaf_rn(pr, A.z, A.x);
  cy = __fmaf_rn(pr, A.w, A.y);
  const float dx = cx - px, dy = cy - py;
  proj = pr;
  return __fmaf_rn(dx, dx, dy * dy);
}

__device__ __forceinline__ float fill_coverage(float md, int w, int n, int rule, float inv_sigma,
                                               float& sign, float& dist) {
  const int inside = (rule == 0) ? (n & 1) : (w != 0);
  dist = sqrtf(fmaxf(md, 0.0f));
  sign = inside ? -1.0f : 1.0f;
  float logit = sign * dist * inv_sigma * 2.0f;
  logit = fmaxf(-60.0f, fminf(60.0f, logit));
  return 1.0f / (1.0f + cs_expf(logit));
}

__device__ __forceinline__ float stroke_coverage(float md, float half_sw, float inv_s2,
                                                 float& dist, float& edge_d) {
  dist = sqrtf(fmaxf(md, 0.0f));
  edge_d = fmaxf(0.0f, dist - half_sw);
  const float sigma = 0.5f * edge_d * edge_d * inv_s2;
  return cs_expf(-sigma);
}

// The backward's coverage: the same formulas with the hardware's fast square
// root, exponential and division (a few ulp; the forward, whose image must
// match the oracle bit for bit, keeps the correctly rounded forms above).
__device__ __forceinline__ float fast_sqrt(float x) {
  return x > 0.0f ? x * rsqrtf(x) : 0.0f;
}

__device__ __forceinline__ float fill_coverage_fast(float md, int w, int n, int rule,
                                                    float inv_sigma, float& sign, float& dist) {
  const int inside = (rule == 0) ? (n & 1) : (w != 0);
  dist = fast_sqrt(md);
  sign = inside ? -1.0f : 1.0f;
  float logit = sign * dist * inv_sigma * 2.0f;
  logit = fmaxf(-60.0f, fminf(60.0f, logit));
  return __fdividef(1.0f, 1.0f + __expf(logit));
}

__device__ __forceinline__ float stroke_coverage_fast(float md, float half_sw, float inv_s2,
                                                      float& dist, float& edge_d) {
  dist = fast_sqrt(md);
  edge_d = fmaxf(0.0f, dist - half_sw);
  const float sigma = 0.5f * edge_d * edge_d * inv_s2;
  return __expf(-sigma);
}

__device__ __forceinline__ void load_meta(const IMeta* __restrict__ p, IMeta& m) {
  const int4* q = reinterpret_cast<const int4*>(p);
  int4 x = __ldg(q), y = __ldg(q + 1), z = __ldg(q + 2);
  m.dstart = x.x; m.dcount = x.y; m.pid = x.z; m.rule = x.w;
  m.c0 = __int_as_float(y.x); m.c1 = __int_as_float(y.y);
  m.c2 = __int_as_float(y.z); m.op = __int_as_float(y.w);
  m.a = __int_as_float(z.x); m.b = __int_as_float(z.y); m.dthr = __int_as_float(z.z);
  m.spare = 0.0f;
}

// ---------------------------------------------------------------------------
// forward

struct FwdPix {
  float T, a0, a1, a2, md;
  int cur, w, n;
  bool done;
  int win;  // closest record of the current intersect, relative to its first
};

// A pixel's code for the backward: bits 0-6 the closest record of the
// intersect relative to its first (127: none or not representable), bit 7
// the pixel's inside/outside state (fills).
constexpr int kNoWinner = 127;
__device__ __forceinline__ unsigned winner_code(int win, bool inside) {
  return (unsigned)(win < kNoWinner ? win : kNoWinner) | (inside ? 128u : 0u);
}

// Squared distances of a lane's two pixels (P = (px0, px1), same row py) to
// the edge of record (A, B): seg_d2's arithmetic on both pixels at once with
// the packed FP32x2 operations of sm_100 (each component rounded exactly as
// the scalar operation: px - x0 is px + (-x0), cx - px is cx + (-px)).
// NP = -P and npy = (-py, -py) are the caller's loop invariants.
__device__ __forceinline__ float2 seg_d2_pair(float2 P, float2 NP, float2 npy, float wy,
                                              const float4& A, const float4& B) {
  const float2 wx = __fadd2_rn(P, make_float2(-A.x, -A.x));
  const float t = wy * A.w;
  float2 pr = __ffma2_rn(wx, make_float2(A.z, A.z), make_float2(t, t));
  pr = __fmul2_rn(pr, make_float2(B.x, B.x));
  pr.x = fmaxf(0.0f, fminf(1.0f, pr.x));
  pr.y = fmaxf(0.0f, fminf(1.0f, pr.y));
  const float2 cx = __ffma2_rn(pr, make_float2(A.z, A.z), make_float2(A.x, A.x));
  const float2 cy = __ffma2_rn(pr, make_float2(A.w, A.w), make_float2(A.y, A.y));
  const float2 dx = __fadd2_rn(cx, NP), dy = __fadd2_rn(cy, npy);
  return __ffma2_rn(dx, dx, __fmul2_rn(dy, dy));
}

template <bool STROKE>
__device__ __forceinline__ void fwd_entries(const DEntry* __restrict__ buf, int c0, int ds, int lo,
                                            int hi, float px0, float px1, float py, FwdPix& p0,
                                            FwdPix& p1) {
  const float2 P = make_float2(px0, px1), NP = make_float2(-px0, -px1);
  const float2 npy = make_float2(-py, -py);
#pragma unroll 2  // two records' distance arithmetic in flight (same order of updates)
  for (int d = lo; d < hi; ++d) {
    const float4 EA = buf[d - c0].a;
    const float4 EB = buf[d - c0].b;
    const float wy = py - EA.y;
    const float2 d2 = seg_d2_pair(P, NP, npy, wy, EA, EB);
    if (!STROKE) {  // the running minimum and its first record (strict <: the first minimum)
      if (d2.x < p0.md) {
        p0.md = d2.x;
        p0.win = d - ds;
      }
      if (d2.y < p1.md) {
        p1.md = d2.y;
        p1.win = d - ds;
      }
    } else {
      p0.md = fminf(p0.md, d2.x);
      p1.md = fminf(p1.md, d2.y);
    }
    if (!STROKE) {
      if (((EA.y <= py) & (EB.y > py)) | ((EA.y > py) & (EB.y <= py))) {
        const float lhs = EB.z + wy * EA.z;
        const float2 rhs = __fmul2_rn(P, make_float2(EA.w, EA.w));
        const bool pos = EA.w > 0.0f;
        const int h0 = pos ? (lhs > rhs.x) : (lhs < rhs.x);
        const int h1 = pos ? (lhs > rhs.y) : (lhs < rhs.y);
        const int sg = pos ? 1 : -1;
        p0.n += h0;
        p1.n += h1;
        p0.w += h0 * sg;
        p1.w += h1 * sg;
      }
    }
  }
}

// Returns whether the pixel composited this intersect (alpha >= alpha_min).
template <bool STROKE>
__device__ __forceinline__ bool fwd_composite(FwdPix& p, const IMeta& m, int k) {
  if (p.done) return false;
  float cov;
  if (!STROKE) {
    float sign, dist;
    cov = fill_coverage(p.md, p.w, p.n, m.rule, m.a, sign, dist);
  } else {
    float dist, edge_d;
    cov = stroke_coverage(p.md, m.b, m.a, dist, edge_d);
  }
  const float alpha = fminf(kAlphaCap, m.op * cov);
  if (alpha < kAlphaMin) return false;
  const float nT = p.T * (1.0f - alpha);
  const float vis = alpha * p.T;
  p.a0 += m.c0 * vis;
  p.a1 += m.c1 * vis;
  p.a2 += m.c2 * vis;
  p.T = nT;
  p.cur = k;
  if (nT <= kTransStop) p.done = true;
  return true;
}

// Forward of one unit by one warp.  Returns false if a bounded wait gave up.
template <bool STROKE>
__device__ __forceinline__ bool forward_unit(const RasterArgs& A, int unit,
                                             DEntry (*buf)[kWChunk], uint64_t* bars,
                                             uint32_t& phase, IBatch& ib, int& work) {
  const int lane = threadIdx.x & 31;
  const UnitGeom g = unit_geom(A, unit);
  const int rs = g.rs, re = g.re, st = g.st;
  const int nd = re > rs ? strip_records_upto(A, re - 1, st) : 0;
  const int nchunks = max(1, (nd + kWChunk - 1) / kWChunk);
  // an empty tile has no list (its bins need not lie between its neighbours')
  int* vl = (A.visits && re > rs) ? A.visits + visit_base(g) : nullptr;
  const int ly = st * kStripRows + (lane >> 3), lx = (lane & 7) * 2;
  const int i = g.ty * kTile + ly, j0 = g.tx * kTile + lx;
  const bool in0 = i < A.H && j0 < A.W, in1 = i < A.H && j0 + 1 < A.W;
  const float py = (float)i + 0.5f;
  const float px0 = (float)j0 + 0.5f, px1 = (float)(j0 + 1) + 0.5f;
  FwdPix p0{1.0f, 0.f, 0.f, 0.f, 1e30f, 0, 0, 0, !in0, kNoWinner};
  FwdPix p1{1.0f, 0.f, 0.f, 0.f, 1e30f, 0, 0, 0, !in1, kNoWinner};
  if (nd > 0 && lane == 0)
    bulk_load(buf[0], A.dl + g.base, (uint32_t)min(nd, kWChunk) * sizeof(DEntry), &bars[0]);
  int k = rs;          // next intersect
  int kb = rs - 32;    // first intersect of the batch in shared memory
  int recs = 0;        // records visited (a work measure for the backward's dispatch)
  int visits = 0;      // intersects that could change a pixel of the strip
  int contrib = 0;     // intersects some pixel of the strip composited
  unsigned amask = 0u; // active intersects of the batch
  bool mid = false;    // k partially visited (split across chunks)
  bool ok = true;
  for (int c = 0; c < nchunks; ++c) {
    const int c0 = c * kWChunk, c1 = min(nd, c0 + kWChunk);
    const bool more = nd > 0 && c + 1 < nchunks;
    if (nd > 0) {
      if (more) {
        __syncwarp();  // every lane is done with the buffer about to be refilled
        if (lane == 0) {
          fence_proxy_async();
          bulk_load(buf[(c + 1) & 1], A.dl + g.base + c1,
                    (uint32_t)min(nd - c1, kWChunk) * sizeof(DEntry), &bars[(c + 1) & 1]);
        }
      }
      ok = wait_buffer(bars, c & 1, phase, A.status);
      if (!ok) break;
    }
    const DEntry* cb = buf[c & 1];  // record d of the strip is cb[d - c0]
    bool finished = false;
    while (k < re) {
      if (!__any_sync(0xffffffffu, !(p0.done && p1.done))) {
        finished = true;
        break;
      }
      if (k >= kb + 32) {
        kb = k;
        amask = load_batch<STROKE>(A, nullptr, kb, min(32, re - kb), st, rs, re, ib);
      }
      const int j = k - kb;
      if (!mid && !((amask >> j) & 1u)) {  // skip to the batch's next active intersect
        const unsigned rest = amask & (0xfffffffeu << j);
        k = rest ? kb + __ffs(rest) - 1 : min(kb + 32, re);
        continue;
      }
      IMeta m;
      batch_meta(ib, j, m);
      const int2 rg = ib.rg[j];
      const int ds = rg.x, de = rg.x + rg.y;
      if (!mid) {
        p0.md = p1.md = 1e30f;
        p0.win = p1.win = kNoWinner;
        p0.w = p0.n = p1.w = p1.n = 0;
      }
      fwd_entries<STROKE>(cb, c0, ds, max(ds, c0), min(de, c1), px0, px1, py, p0, p1);
      recs += max(0, min(de, c1) - max(ds, c0));
      if (de > c1) {
        mid = true;
        break;
      }
      if (!STROKE) {
        const int ro = batch_rowoff(ib, j);
        const int rw = row_wind(ro), rc = row_cnt(ro);
        p0.w += rw; p1.w += rw; p0.n += rc; p1.n += rc;
      }
      const bool c0 = fwd_composite<STROKE>(p0, m, k);
      const bool c1 = fwd_composite<STROKE>(p1, m, k);
      if (__any_sync(0xffffffffu, c0 || c1)) {
        if (vl && lane == 0) vl[1 + contrib] = k;
        if (!STROKE && vl && A.winners) {  // this visit's closest records, for the backward
          const bool i0 = m.rule == 0 ? (p0.n & 1) != 0 : p0.w != 0;
          const bool i1 = m.rule == 0 ? (p1.n & 1) != 0 : p1.w != 0;
          A.winners[(visit_base(g) + 1 + contrib) * 32 + lane] =
              (unsigned short)(winner_code(p0.win, i0) | (winner_code(p1.win, i1) << 8));
        }
        ++contrib;
      }
      ++visits;
      mid = false;
      ++k;
    }
    if (finished || k >= re) {
      if (more) {  // drain the prefetched chunk before the buffer is reused
        ok = wait_buffer(bars, (c + 1) & 1, phase, A.status);
      }
      break;
    }
  }
  __syncwarp();  // the buffers are free for the next unit
  const float bg0 = A.bg[0], bg1 = A.bg[1], bg2 = A.bg[2];
  const long long hw = (long long)A.H * A.W;
  float sse = 0.0f;
  if (ok && A.vec2 && in0 && in1) {  // both pixels: paired 8-byte stores and loads
    const long long pix = (long long)i * A.W + j0;
    const float o[2][3] = {{p0.a0 + p0.T * bg0, p0.a1 + p0.T * bg1, p0.a2 + p0.T * bg2},
                           {p1.a0 + p1.T * bg0, p1.a1 + p1.T * bg1, p1.a2 + p1.T * bg2}};
    *reinterpret_cast<float2*>(A.fts + pix) = make_float2(p0.T, p1.T);
    *reinterpret_cast<int2*>(A.fidx + pix) = make_int2(p0.cur, p1.cur);
    float2* oh = reinterpret_cast<float2*>(A.out + pix * 3);
    oh[0] = make_float2(o[0][0], o[0][1]);
    oh[1] = make_float2(o[0][2], o[1][0]);
    oh[2] = make_float2(o[1][1], o[1][2]);
    float kc[2][3];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int c = 0; c < 3; ++c) kc[u][c] = fminf(fmaxf(o[u][c], 0.0f), 1.0f);
    if (A.out_chw) {
#pragma unroll
      for (int c = 0; c < 3; ++c)
        *reinterpret_cast<float2*>(A.out_chw + c * hw + pix) = make_float2(kc[0][c], kc[1][c]);
    }
    if (A.loss_tgt) {
      float2 t[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) t[c] = *reinterpret_cast<const float2*>(A.loss_tgt + c * hw + pix);
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float d = kc[0][c] - t[c].x;
        sse = __fmaf_rn(d, d, sse);
      }
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float d = kc[1][c] - t[c].y;
        sse = __fmaf_rn(d, d, sse);
      }
    }
  } else {
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const FwdPix& p = u ? p1 : p0;
    if (!ok || !(u ? in1 : in0)) continue;
    const long long pix = (long long)i * A.W + j0 + u;
    const float o0 = p.a0 + p.T * bg0, o1 = p.a1 + p.T * bg1, o2 = p.a2 + p.T * bg2;
    A.fts[pix] = p.T;
    A.fidx[pix] = p.cur;
    A.out[pix * 3] = o0;
    A.out[pix * 3 + 1] = o1;
    A.out[pix * 3 + 2] = o2;
    const float k0 = fminf(fmaxf(o0, 0.0f), 1.0f), k1 = fminf(fmaxf(o1, 0.0f), 1.0f),
                k2 = fminf(fmaxf(o2, 0.0f), 1.0f);
    if (A.out_chw) {
      A.out_chw[pix] = k0;
      A.out_chw[hw + pix] = k1;
      A.out_chw[2 * hw + pix] = k2;
    }
    if (A.loss_tgt) {
      const float d0 = k0 - A.loss_tgt[pix], d1 = k1 - A.loss_tgt[hw + pix],
                  d2 = k2 - A.loss_tgt[2 * hw + pix];
      sse = __fmaf_rn(d0, d0, sse);
      sse = __fmaf_rn(d1, d1, sse);
      sse = __fmaf_rn(d2, d2, sse);
    }
  }
  }
  if (A.loss_tgt) {
    sse = warp_sum(sse);
    if (lane == 0) A.partials[unit] = sse;  // indexed by unit: a fixed reduction order
  }
  if (vl && lane == 0) vl[0] = contrib;
  // the backward visits about the same intersects and records, and runs the
  // gradient arithmetic for the whole warp where any pixel composited
  work = k > rs ? 2 * recs + 4 * (visits + (k < re ? 1 : 0)) + 10 * contrib + (k - rs) / 4 : 0;
  return ok;
}

template <bool STROKE>
__global__ void __launch_bounds__(kRT) raster_forward_kernel(const RasterArgs A) {
  __shared__ __align__(128) DEntry sbuf[kRW][2][kWChunk];
  __shared__ __align__(16) IBatch sib[kRW];
  __shared__ __align__(8) uint64_t sbar[kRW][2];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint64_t* bars = sbar[wid];
  if (lane == 0) {
    mbar_init(&bars[0]);
    mbar_init(&bars[1]);
    fence_barrier_init();
  }
  __syncwarp();  // the warp's barriers are initialised before anyone waits on them
  uint32_t phase = 0u;  // bit b: parity of the next completion of buffer b's barrier
  int pre0 = 0, pre1 = 0;
  if (A.order) unit_prefix(A.order, pre0, pre1);
  int u = blockIdx.x * kRW + wid;
  while (u < A.nunits) {
    const int unit = A.order ? unit_at(A.order, A.nunits, u, pre0, pre1) : u;
    if ((unsigned)unit >= (unsigned)A.nunits) {  // malformed dispatch lists
      if (lane == 0 && A.status) atomicExch(A.status, CS_ERR_ARG);
      break;
    }
    int work = 0;
    const bool ok = forward_unit<STROKE>(A, unit, sbuf[wid], bars, phase, sib[wid], work);
    if (A.order_next && lane == 0) append_unit(A.order_next, A.nunits, unit, work);
    if (!ok) break;
    u = next_unit(A);
  }
  finish_launch(A, A.loss_tgt != nullptr);
}

// ---------------------------------------------------------------------------
// backward

struct BwdPix {
  float T, Tf, b0, b1, b2, v0, v1, v2, bgd;
  int fidx;
  bool in;
  float md, bp, bcx, bcy;
  int be, bl, w, n;  // bl: staged record of the closest edge in the current chunk, or -1
};

// Closest record of the intersect so far and the crossing counts.  Records of
// an intersect lie in edge order, so while they are visited in order a strict
// < keeps the reference's first minimum.  An intersect whose records span
// staging chunks is visited chunk by chunk from the top; in every chunk after
// the first (TIES) an equal distance goes to the lower edge id explicitly.
// Only the distance and the record index are tracked here; the closest point
// of the winner is recomputed once per intersect (best_point).
template <bool STROKE, bool TIES>
__device__ __forceinline__ void bwd_entries(const DEntry* __restrict__ buf, int c0, int lo, int hi,
                                            const float px[2], float py, BwdPix s[2]) {
  const float2 P = make_float2(px[0], px[1]), NP = make_float2(-px[0], -px[1]);
  const float2 npy = make_float2(-py, -py);
  for (int d = lo; d < hi; ++d) {
    const float4 EA = buf[d - c0].a;
    const float4 EB = buf[d - c0].b;
    const float wy = py - EA.y;
    const float2 dd = seg_d2_pair(P, NP, npy, wy, EA, EB);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float d2 = u ? dd.y : dd.x;
      bool take = d2 < s[u].md;
      if (TIES) {
        const int eid = __float_as_int(EB.w);
        take = take || (d2 == s[u].md && eid < s[u].be);
        if (take) s[u].be = eid;
      }
      if (take) {
        s[u].md = d2;
        s[u].bl = d;
      }
    }
    if (!STROKE) {
      if (((EA.y <= py) & (EB.y > py)) | ((EA.y > py) & (EB.y <= py))) {
        const float lhs = EB.z + wy * EA.z;
        const bool pos = EA.w > 0.0f;
        const int sg = pos ? 1 : -1;
        const float2 rr = __fmul2_rn(P, make_float2(EA.w, EA.w));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float rhs = u ? rr.y : rr.x;
          const int h = pos ? (lhs > rhs) : (lhs < rhs);
          s[u].n += h;
          s[u].w += h * sg;
        }
      }
    }
  }
}

// Projection, closest point and edge id of the pixel's closest record, which
// must be resident in the current chunk (bl >= 0).
__device__ __forceinline__ void best_point(const DEntry* __restrict__ buf, int c0, float px,
                                           float py, BwdPix& s) {
  const float4 EA = buf[s.bl - c0].a;
  const float4 EB = buf[s.bl - c0].b;
  s.be = __float_as_int(EB.w);
  seg_d2(px, py, py - EA.y, EA, EB, s.bp, s.bcx, s.bcy);
}

// One pixel's backward step at one intersect.  need_op / need_inv say whether
// the opacity and softness gradients are wanted at all (NULL outputs skip
// their arithmetic).  Uses the fast coverage and reciprocal forms: the
// gradients only need to match the reference within its tolerance.
template <bool STROKE>
__device__ __forceinline__ void bwd_pixel(BwdPix& s, const IMeta& m, float px, float py, bool valid,
                                          float acc[kAcc], bool collect, bool need_op,
                                          bool need_inv, float4& eg, bool& has_eg,
                                          bool& contributed) {
  has_eg = false;
  if (!valid) return;
  float cov, sign = 1.0f, dist, edge_d = 0.0f;
  if (!STROKE) {
    cov = fill_coverage_fast(s.md, s.w, s.n, m.rule, m.a, sign, dist);
  } else {
    cov = stroke_coverage_fast(s.md, m.b, m.a, dist, edge_d);
  }
  const float op = m.op;
  const float alpha = fminf(kAlphaCap, op * cov);
  if (!(alpha >= kAlphaMin)) return;
  contributed = true;
  const float ra = __fdividef(1.0f, 1.0f - alpha);
  s.T = s.T * ra;
  const float fac = alpha * s.T;
  acc[0] += fac * s.v0;
  acc[1] += fac * s.v1;
  acc[2] += fac * s.v2;
  if (collect) {
    const float c0 = fac * m.c0, c1 = fac * m.c1, c2 = fac * m.c2;
    acc[6] += c0;
    acc[7] += c1;
    acc[8] += c2;
    acc[9] += c0 + c1 + c2;
  }
  float v_alpha = 0.0f;
  v_alpha = v_alpha + (m.c0 * s.T - s.b0 * ra) * s.v0;
  v_alpha = v_alpha + (m.c1 * s.T - s.b1 * ra) * s.v1;
  v_alpha = v_alpha + (m.c2 * s.T - s.b2 * ra) * s.v2;
  v_alpha = v_alpha + s.Tf * ra * (0.0f - s.bgd);
  s.b0 = s.b0 + m.c0 * fac;
  s.b1 = s.b1 + m.c1 * fac;
  s.b2 = s.b2 + m.c2 * fac;
  if (!(alpha < kAlphaCap)) return;
  if (need_op) acc[3] += cov * v_alpha;
  float gscale = 0.0f;
  bool geom = false;
  if (!STROKE) {
    const float v_cov = op * v_alpha;
    const float v_logit = -v_cov * cov * (1.0f - cov);
    if (need_inv) {
      const float v_inv_sigma = v_logit * sign * dist * 2.0f;
      acc[4] += __fdividef(v_inv_sigma * 0.5f, fmaxf(m.a, kEps));
    }
    gscale = v_logit * sign * m.a * 2.0f;
    geom = (dist > kEps) & (s.be >= 0);
  } else {
    const float v_sigma = -op * cov * v_alpha;
    if (need_inv) acc[4] += 0.5f * edge_d * edge_d * v_sigma;
    if (edge_d > 0.0f) {
      const float v_edge = v_sigma * edge_d * m.a;
      acc[5] += -0.5f * v_edge;
      gscale = v_edge;
      geom = (dist > kEps) & (s.be >= 0);
    }
  }
  if (geom) {
    const float g = __fdividef(gscale, dist);  // gscale / dist, once for both axes
    const float gx = g * (s.bcx - px);
    const float gy = g * (s.bcy - py);
    eg = make_float4((1.0f - s.bp) * gx, (1.0f - s.bp) * gy, s.bp * gx, s.bp * gy);
    has_eg = true;
  }
}

// Warp totals of four values at once (two exchange rounds that halve the
// values each lane carries, then three plain rounds): returns, in every lane,
// the total of value ((lane >> 3) & 3).  Six shuffles instead of twenty.
__device__ __forceinline__ float warp_reduce4(float v0, float v1, float v2, float v3) {
  const int lane = threadIdx.x & 31;
  const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
  float a = h16 ? v2 : v0, b = h16 ? v3 : v1;
  a += __shfl_xor_sync(0xffffffffu, h16 ? v0 : v2, 16);
  b += __shfl_xor_sync(0xffffffffu, h16 ? v1 : v3, 16);
  float c = h8 ? b : a;
  c += __shfl_xor_sync(0xffffffffu, h8 ? a : b, 8);
  c += __shfl_xor_sync(0xffffffffu, c, 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

// Edge-endpoint gradients of one visit.  Many pixels of a strip share a
// winner edge, and per-pixel atomics on one address serialise, so the warp
// first sums its contributions per distinct winner -- one ballot round and one
// four-value butterfly per winner -- and then four lanes add the four
// components.  key >= 0: the winner's record is resident, the sum goes to the
// chunk's shared accumulator dgrad[key - c0]; key = -(edge + 2): its record
// is no longer resident, the sum goes to v_edges directly.
__device__ __forceinline__ void add_edge_grads(const RasterArgs& A, float4* dgrad, int c0,
                                               int key0, bool has0, const float4& g0, int key1,
                                               bool has1, const float4& g1) {
  const int lane = threadIdx.x & 31;
  unsigned p0 = __ballot_sync(0xffffffffu, has0), p1 = __ballot_sync(0xffffffffu, has1);
  while (p0 | p1) {  // every round clears at least the source lane's bit
    const int src = p0 ? __ffs(p0) - 1 : __ffs(p1) - 1;
    const int k = __shfl_sync(0xffffffffu, p0 ? key0 : key1, src);
    const bool m0 = has0 && key0 == k, m1 = has1 && key1 == k;
    p0 &= ~__ballot_sync(0xffffffffu, m0);
    p1 &= ~__ballot_sync(0xffffffffu, m1);
    float x = 0.0f, y = 0.0f, z = 0.0f, w = 0.0f;
    if (m0) { x = g0.x; y = g0.y; z = g0.z; w = g0.w; }
    if (m1) { x += g1.x; y += g1.y; z += g1.z; w += g1.w; }
    const float r = warp_reduce4(x, y, z, w);
    if ((lane & 7) == 0 && r != 0.0f) {
      const int vi = lane >> 3;
      if (k >= 0)
        atomicAdd(reinterpret_cast<float*>(dgrad + (k - c0)) + vi, r);
      else
        atomicAdd(A.v_edges + (long long)(-(k + 2)) * 4 + vi, r);
    }
  }
}

__device__ __forceinline__ void flush_acc(const RasterArgs& A, int pid, int k, int c, float v) {
  if (v == 0.0f) return;
  if (c < 3) atomicAdd(A.v_colors + pid * 3 + c, v);
  else if (c == 3) { if (A.v_opac) atomicAdd(A.v_opac + pid, v); }
  else if (c == 4) { if (A.v_inv) atomicAdd(A.v_inv + pid, v); }
  else if (c == 5) atomicAdd(A.v_sw + pid, v);
  else if (c < 9) { if (A.contrib) atomicAdd(A.contrib + pid * 3 + (c - 6), v); }
  else if (A.icontrib) atomicAdd(A.icontrib + k, v);
}

// Sums over the warp of eight values at once: on return lane l holds the
// total of value l / 4 (a reduce-scatter: four, two and one exchanged values,
// then two butterfly steps).
__device__ __forceinline__ float warp_reduce8(const float v[8]) {
  const int lane = threadIdx.x & 31;
  const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0, h4 = (lane & 4) != 0;
  float a[4], b[2];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    a[i] = (h16 ? v[4 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, h16 ? v[i] : v[4 + i], 16);
#pragma unroll
  for (int i = 0; i < 2; ++i)
    b[i] = (h8 ? a[2 + i] : a[i]) + __shfl_xor_sync(0xffffffffu, h8 ? a[i] : a[2 + i], 8);
  float c = (h4 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, h4 ? b[0] : b[1], 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

// add_edge_grads for the direct backward (every sum goes to v_edges; key =
// -(edge + 2)), two distinct winners per round when there are two: their
// eight components share one reduce-scatter, so a visit with several winner
// edges needs half the dependent shuffle rounds.  With `fold` (warp-uniform)
// the visit's four per-primitive sums (colours, opacity) ride in the free half
// of a last round that has a single winner, and the function returns true
// once it has flushed them (else the caller reduces them itself).
__device__ __forceinline__ bool add_edge_grads_direct(const RasterArgs& A, int key0, bool has0,
                                                      const float4& g0, int key1, bool has1,
                                                      const float4& g1, bool fold,
                                                      const float a4[4], int pid, int k) {
  const int lane = threadIdx.x & 31;
  unsigned p0 = __ballot_sync(0xffffffffu, has0), p1 = __ballot_sync(0xffffffffu, has1);
  while (p0 | p1) {  // every round clears at least the source lane's bit
    const int sa = p0 ? __ffs(p0) - 1 : __ffs(p1) - 1;
    const int ka = __shfl_sync(0xffffffffu, p0 ? key0 : key1, sa);
    const bool a0 = has0 && key0 == ka, a1 = has1 && key1 == ka;
    p0 &= ~__ballot_sync(0xffffffffu, a0);
    p1 &= ~__ballot_sync(0xffffffffu, a1);
    float v[8];
    v[0] = v[1] = v[2] = v[3] = 0.0f;
    if (a0) { v[0] = g0.x; v[1] = g0.y; v[2] = g0.z; v[3] = g0.w; }
    if (a1) { v[0] += g1.x; v[1] += g1.y; v[2] += g1.z; v[3] += g1.w; }
    if (!(p0 | p1)) {  // one winner left
      if (fold) {
        v[4] = a4[0];
        v[5] = a4[1];
        v[6] = a4[2];
        v[7] = a4[3];
        const float r = warp_reduce8(v);
        const int vi = lane >> 2;
        if ((lane & 3) == 0 && r != 0.0f) {
          if (vi < 4)
            atomicAdd(A.v_edges + (long long)(-(ka + 2)) * 4 + vi, r);
          else
            flush_acc(A, pid, k, vi - 4, r);
        }
        return true;
      }
      const float r = warp_reduce4(v[0], v[1], v[2], v[3]);
      if ((lane & 7) == 0 && r != 0.0f)
        atomicAdd(A.v_edges + (long long)(-(ka + 2)) * 4 + (lane >> 3), r);
      return false;
    }
    const int sb = p0 ? __ffs(p0) - 1 : __ffs(p1) - 1;
    const int kb = __shfl_sync(0xffffffffu, p0 ? key0 : key1, sb);
    const bool b0 = has0 && key0 == kb, b1 = has1 && key1 == kb;
    p0 &= ~__ballot_sync(0xffffffffu, b0);
    p1 &= ~__ballot_sync(0xffffffffu, b1);
    v[4] = v[5] = v[6] = v[7] = 0.0f;
    if (b0) { v[4] = g0.x; v[5] = g0.y; v[6] = g0.z; v[7] = g0.w; }
    if (b1) { v[4] += g1.x; v[5] += g1.y; v[6] += g1.z; v[7] += g1.w; }
    const float r = warp_reduce8(v);
    const int vi = lane >> 2;
    if ((lane & 3) == 0 && r != 0.0f)
      atomicAdd(A.v_edges + (long long)(-((vi < 4 ? ka : kb) + 2)) * 4 + (vi & 3), r);
  }
  return false;
}


// Per-pixel state of a backward strip: T, final_idx and the image gradient
// (given, or the MSE gradient from the image and the target), with paired
// 8-byte loads when both pixels are in the image.  Returns the warp's last
// needed intersect (the largest final_idx, at most re - 1).
__device__ __forceinline__ int bwd_setup(const RasterArgs& A, int i, int j0, int re,
                                         BwdPix s[2]) {
  const float scale = A.v_out ? 0.0f : *A.mse_scale;
  int kmax = -1;
  const bool in2[2] = {i < A.H && j0 < A.W, i < A.H && j0 + 1 < A.W};
  float T2[2] = {1.0f, 1.0f}, vv[2][3] = {{0.f, 0.f, 0.f}, {0.f, 0.f, 0.f}};
  int F2[2] = {-1, -1};
  const long long hw = (long long)A.H * A.W;
  const long long pix0 = (long long)i * A.W + j0;
  if (A.vec2 && in2[0] && in2[1]) {
    const float2 t2 = *reinterpret_cast<const float2*>(A.fts_in + pix0);
    const int2 f2 = *reinterpret_cast<const int2*>(A.fidx_in + pix0);
    T2[0] = t2.x; T2[1] = t2.y; F2[0] = f2.x; F2[1] = f2.y;
    const float2* src = reinterpret_cast<const float2*>((A.v_out ? A.v_out : A.out_img) + pix0 * 3);
    const float2 a = src[0], b = src[1], c = src[2];
    const float o[2][3] = {{a.x, a.y, b.x}, {b.y, c.x, c.y}};
    if (A.v_out) {
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) vv[u][ch] = o[u][ch];
    } else {
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        const float2 t = *reinterpret_cast<const float2*>(A.tgt + ch * hw + pix0);
        vv[0][ch] = (o[0][ch] >= 0.0f && o[0][ch] <= 1.0f) ? scale * (o[0][ch] - t.x) : 0.0f;
        vv[1][ch] = (o[1][ch] >= 0.0f && o[1][ch] <= 1.0f) ? scale * (o[1][ch] - t.y) : 0.0f;
      }
    }
  } else {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!in2[u]) continue;
      const long long pix = pix0 + u;
      T2[u] = A.fts_in[pix];
      F2[u] = A.fidx_in[pix];
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        if (A.v_out) {
          vv[u][ch] = A.v_out[pix * 3 + ch];
        } else {
          const float o = A.out_img[pix * 3 + ch];
          const float t = A.tgt[ch * hw + pix];
          vv[u][ch] = (o >= 0.0f && o <= 1.0f) ? scale * (o - t) : 0.0f;
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    s[u].in = in2[u];
    s[u].b0 = s[u].b1 = s[u].b2 = 0.0f;
    s[u].md = 1e30f;
    s[u].be = -1;
    s[u].bl = -1;
    s[u].bp = s[u].bcx = s[u].bcy = 0.0f;
    s[u].w = s[u].n = 0;
    s[u].T = T2[u];
    s[u].fidx = F2[u];
    s[u].v0 = vv[u][0];
    s[u].v1 = vv[u][1];
    s[u].v2 = vv[u][2];
    s[u].bgd = in2[u] ? A.bg[0] * vv[u][0] + A.bg[1] * vv[u][1] + A.bg[2] * vv[u][2] : 0.0f;
    if (in2[u]) kmax = max(kmax, s[u].fidx);
    s[u].Tf = s[u].T;
  }
  return min(warp_max_i(kmax), re - 1);  // this warp's last needed intersect
}

// Backward of one unit by one warp.  Returns false if a bounded wait gave up.
template <bool STROKE>
__device__ __forceinline__ bool backward_unit(const RasterArgs& A, int unit,
                                              DEntry (*buf)[kWChunk], uint64_t* bars,
                                              uint32_t& phase, float4* dgrad, IBatch& ib) {
  const int lane = threadIdx.x & 31;
  const UnitGeom g = unit_geom(A, unit);
  const int rs = g.rs, re = g.re, st = g.st;
  if (re <= rs) return true;
  const int ly = st * kStripRows + (lane >> 3), lx = (lane & 7) * 2;
  const int i = g.ty * kTile + ly, j0 = g.tx * kTile + lx;
  const float py = (float)i + 0.5f;
  const float px[2] = {(float)j0 + 0.5f, (float)(j0 + 1) + 0.5f};
  const bool collect = (A.contrib != nullptr) | (A.icontrib != nullptr);
  BwdPix s[2];
  int kmax = bwd_setup(A, i, j0, re, s);
  if (kmax < rs) return true;
  // The walk runs over positions q = nq - 1 .. 0: every intersect rs .. kmax
  // (position q is intersect rs + q), or the forward's list of the strip's
  // intersects that composited a pixel (no other intersect changes a pixel's
  // T or gets a gradient: a pixel composites k exactly when alpha_k >=
  // alpha_min and k <= final_idx).
  const int* vl = nullptr;
  long long wslot = 0;  // visit-list slot of position 0 (for the winner codes)
  int nq = kmax - rs + 1;
  if (A.visits) {
    vl = A.visits + visit_base(g);
    const int cnt = vl[0];
    if (cnt < 0 || cnt > re - rs) {  // not a list the forward wrote for this strip
      if (lane == 0 && A.status) atomicExch(A.status, CS_ERR_ARG);
      return true;
    }
    ++vl;
    nq = cnt;
    wslot = visit_base(g) + 1;
    if (nq == 0) return true;
    const int klast = vl[nq - 1];
    if (klast >= rs && klast < kmax) kmax = klast;  // fewer record chunks to bring in
  }
  const int nd = strip_records_upto(A, kmax, st);  // records of intersects <= kmax
  const int nchunks = max(1, (nd + kWChunk - 1) / kWChunk);
  const int last = nchunks - 1;
  if (nd > 0 && lane == 0) {
    const int c0 = last * kWChunk;
    bulk_load(buf[last & 1], A.dl + g.base + c0, (uint32_t)(nd - c0) * sizeof(DEntry),
              &bars[last & 1]);
  }
  int q = nq - 1;     // next position (walking down)
  int qb = nq;        // first position of the batch in shared memory (batch: qb .. qb + 31)
  unsigned amask = 0u;  // active intersects of the batch
  bool mid = false;   // the intersect at q partially visited
  bool ok = true;
  for (int c = last; c >= 0; --c) {
    const int c0 = c * kWChunk, c1 = min(nd, c0 + kWChunk);
    const bool more = nd > 0 && c > 0;
    if (nd > 0) {
      if (more) {
        __syncwarp();  // every lane is done with the buffer about to be refilled
        if (lane == 0) {
          fence_proxy_async();
          bulk_load(buf[(c - 1) & 1], A.dl + g.base + (c - 1) * kWChunk,
                    (uint32_t)kWChunk * sizeof(DEntry), &bars[(c - 1) & 1]);
        }
      }
      ok = wait_buffer(bars, c & 1, phase, A.status);
      if (!ok) break;
    }
    const DEntry* cb = buf[c & 1];  // record d of the strip is cb[d - c0]
    while (q >= 0) {
      if (q < qb) {
        qb = max(0, q - 31);
        amask = load_batch<STROKE>(A, vl ? vl + qb : nullptr, rs + qb, q - qb + 1, st, rs, re, ib);
      }
      const int j = q - qb;
      if (!mid && !((amask >> j) & 1u)) {  // skip to the batch's next lower active intersect
        const unsigned below = amask & ((1u << j) - 1u);
        q = below ? qb + 31 - __clz(below) : qb - 1;
        continue;
      }
      const int k = ib.kk[j];
      const bool v0 = s[0].in && k <= s[0].fidx;
      const bool v1 = s[1].in && k <= s[1].fidx;
      IMeta m;
      batch_meta(ib, j, m);
      const int2 rg = ib.rg[j];
      const int ds = rg.x, de = rg.x + rg.y;
      if (!mid) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          s[u].md = 1e30f;
          s[u].be = -1;
          s[u].bl = -1;
          s[u].bp = s[u].bcx = s[u].bcy = 0.0f;
          s[u].w = s[u].n = 0;
        }
      }
      if (de > ds && de <= c0) break;  // its records lie in a lower chunk
      // The forward's closest record and inside state of each pixel of this
      // visit (winner codes): only the winner record is evaluated.  Any
      // pixel that needs the walk (no representable code) sends the warp down
      // the record walk below.
      bool fast = false;
      unsigned wc = 0u;
      if (!STROKE && A.winners && vl && !mid) {
        wc = __ldg(A.winners + (wslot + q) * 32 + lane);
        const bool need0 = v0 && de > ds && (wc & 127u) == kNoWinner;
        const bool need1 = v1 && de > ds && ((wc >> 8) & 127u) == kNoWinner;
        fast = !__any_sync(0xffffffffu, need0 || need1);
      }
      if (fast) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const unsigned c = (wc >> (8 * u)) & 255u;
          const int win = (int)(c & 127u);
          s[u].w = s[u].n = (int)(c >> 7);
          if (win == kNoWinner || de <= ds) continue;
          if (win >= de - ds) {  // not a code the forward wrote for this intersect
            if (A.status) atomicExch(A.status, CS_ERR_ARG);
            continue;
          }
          const int d = ds + win;
          const bool res = d >= c0 && d < c1;  // record in the resident chunk
          float4 EA, EB;
          if (res) {
            EA = cb[d - c0].a;
            EB = cb[d - c0].b;
          } else {
            EA = __ldg(&A.dl[g.base + d].a);
            EB = __ldg(&A.dl[g.base + d].b);
          }
          s[u].md = seg_d2(px[u], py, py - EA.y, EA, EB, s[u].bp, s[u].bcx, s[u].bcy);
          s[u].be = __float_as_int(EB.w);
          s[u].bl = res ? d : -2;
        }
      } else {
        if (mid)
          bwd_entries<STROKE, true>(cb, c0, max(ds, c0), min(de, c1), px, py, s);
        else
          bwd_entries<STROKE, false>(cb, c0, max(ds, c0), min(de, c1), px, py, s);
        // the winner so far, while its record is resident; bl = -2 marks a
        // winner from a chunk that is no longer resident (bp, bcx, bcy, be hold it)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (s[u].bl >= 0) {
            best_point(cb, c0, px[u], py, s[u]);
            if (ds < c0) s[u].bl = -2;
          }
        }
        if (ds < c0) {
          mid = true;
          break;
        }
        if (!STROKE) {
          const int ro = batch_rowoff(ib, j);
          const int rw = row_wind(ro), rc = row_cnt(ro);
          s[0].w += rw; s[1].w += rw; s[0].n += rc; s[1].n += rc;
        }
      }
      float acc[kAcc];
#pragma unroll
      for (int a = 0; a < kAcc; ++a) acc[a] = 0.0f;
      bool contributed = false;
      float4 eg[2];
      bool has_eg[2];
#pragma unroll
      for (int u = 0; u < 2; ++u)
        bwd_pixel<STROKE>(s[u], m, px[u], py, u ? v1 : v0, acc, collect, A.v_opac != nullptr,
                          A.v_inv != nullptr, eg[u], has_eg[u], contributed);
      add_edge_grads(A, dgrad, c0, s[0].bl >= 0 ? s[0].bl : -(s[0].be + 2), has_eg[0], eg[0],
                     s[1].bl >= 0 ? s[1].bl : -(s[1].be + 2), has_eg[1], eg[1]);
      if (__any_sync(0xffffffffu, contributed)) {
        // four sums per butterfly: lane 8 i holds value i's warp total
        const int vi = (lane >> 3) & 3;
        const bool leader = (lane & 7) == 0;
        float r = warp_reduce4(acc[0], acc[1], acc[2], A.v_opac ? acc[3] : 0.0f);
        if (leader) flush_acc(A, m.pid, k, vi, r);
        if (STROKE || A.v_inv) {
          r = warp_reduce4(acc[4], STROKE ? acc[5] : 0.0f, 0.0f, 0.0f);
          if (leader && vi < 2) flush_acc(A, m.pid, k, 4 + vi, r);
        }
        if (collect) {
          r = warp_reduce4(acc[6], acc[7], acc[8], acc[9]);
          if (leader) flush_acc(A, m.pid, k, 6 + vi, r);
        }
      }
      mid = false;
      --q;
    }
    __syncwarp();
    // flush this chunk's edge gradients while its records are resident
    for (int d = c0 + lane; d < c1; d += 32) {
      const float4 gv = dgrad[d - c0];
      if (gv.x == 0.0f && gv.y == 0.0f && gv.z == 0.0f && gv.w == 0.0f) continue;
      float* dst = A.v_edges + (long long)__float_as_int(cb[d - c0].b.w) * 4;
      atomicAdd(dst, gv.x);
      atomicAdd(dst + 1, gv.y);
      atomicAdd(dst + 2, gv.z);
      atomicAdd(dst + 3, gv.w);
      dgrad[d - c0] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncwarp();
    if (q < 0) {
      if (more) {  // drain the prefetched chunk before the buffer is reused
        ok = wait_buffer(bars, (c - 1) & 1, phase, A.status);
      }
      break;
    }
  }
  __syncwarp();
  return ok;
}

// Per-warp shared state of the direct fill backward beside its intersect
// batch: the batch's winner codes (32 positions x 32 lanes, two 8-bit codes
// per lane) and, in two alternating slots, each lane's two pixels' winning
// records of the current and the next visit.
struct DirectBuf {
  unsigned short codes[32 * 32];
  float4 ra[2][2][32];  // [slot][pixel][lane]: the records' two halves apart, so
  float4 rb[2][2][32];  // that a warp's 16-byte reads hit consecutive addresses
};

// Starts the copies of the winner codes of batch positions 0 .. n - 1 (64
// bytes each, contiguous from src) into the warp's shared codes.
__device__ __forceinline__ void stage_codes(const unsigned short* src, int n, DirectBuf& db) {
  const int lane = threadIdx.x & 31;
  for (int c = lane; c < n * 4; c += 32) cp_async16_cg(db.codes + c * 8, src + c * 8);
  cp_async_commit();
}

// Starts the copies of this lane's two pixels' winning records of batch entry
// j into db.ra / db.rb [slot][pixel][lane]: pixels that the visit skips, codes that call for the
// record walk and codes out of the intersect's range copy nothing (they are
// handled, or reported, when the visit is evaluated).
__device__ __forceinline__ void prefetch_winners(const DEntry* dl, const IBatch& ib, int j,
                                                 const BwdPix s[2], DirectBuf& db, int slot) {
  const int lane = threadIdx.x & 31;
  const int k = ib.kk[j];
  const int2 rg = ib.rg[j];
  const unsigned wc = db.codes[j * 32 + lane];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int win = (int)((wc >> (8 * u)) & 127u);
    if (rg.y > 0 && s[u].in && k <= s[u].fidx && win != kNoWinner && win < rg.y) {
      const DEntry* e = dl + rg.x + win;
      cp_async16_ca(&db.ra[slot][u][lane], &e->a);
      cp_async16_ca(&db.rb[slot][u][lane], &e->b);
    }
  }
  cp_async_commit();
}

// Fill backward of one unit from the forward's visit list and winner codes,
// with nothing staged: every listed visit evaluates, per pixel, only the
// closest record the forward found (the records of one intersect sit
// together), and the warp's edge-gradient sums per distinct winner go straight
// to v_edges.  An edge record belongs to one intersect, so a strip visits it
// at most once and a shared accumulator would save no atomics.  A pixel
// without a representable code (an intersect with more than 127 records in
// the strip) walks that intersect's records in order (strict <: the
// reference's first minimum); the code's inside bit holds the pixel's
// crossing state either way.
//
// Memory latency is taken off the per-visit chain: a batch's winner codes are
// copied into shared memory while its intersect records load, and the
// winning records of the next visit of the batch are copied (cp.async) while
// the current visit computes, so a visit waits on memory only when it is the
// first of its batch.
__device__ __forceinline__ bool backward_unit_direct(const RasterArgs& A, int unit, IBatch& ib,
                                                     DirectBuf& db) {
  const int lane = threadIdx.x & 31;
  // the tile's intersect and record ranges and the strip's pixel state are
  // loaded together: one memory round trip instead of three
  UnitGeom g;
  {
    const int trel = unit / kStrips;
    g.st = unit - trel * kStrips;
    const int ry = trel / A.tbx;
    g.tx = trel - ry * A.tbx;
    g.ty = A.r0 + ry;
    g.tile = (long long)g.ty * A.tbx + g.tx;
  }
  g.rs = __ldg(A.bins + 2 * g.tile);
  g.re = __ldg(A.bins + 2 * g.tile + 1);
  const int2 tdl = A.dlr[g.tile];
  const int st = g.st;
  const int ly = st * kStripRows + (lane >> 3), lx = (lane & 7) * 2;
  const int i = g.ty * kTile + ly, j0 = g.tx * kTile + lx;
  const float py = (float)i + 0.5f;
  const float px[2] = {(float)j0 + 0.5f, (float)(j0 + 1) + 0.5f};
  const bool collect = (A.contrib != nullptr) | (A.icontrib != nullptr);
  BwdPix s[2];
  const int kall = bwd_setup(A, i, j0, INT_MAX, s);  // the warp's largest final_idx
  const int rs = g.rs, re = g.re;
  if (re <= rs) return true;
  g.base = (long long)tdl.x + (long long)st * tdl.y;
  const int kmax = min(kall, re - 1);
  if (kmax < rs) return true;
  const int* vl = A.visits + visit_base(g);
  const int cnt = vl[0];
  // the list's first 32 ids come with its count (they are the only batch of a
  // list of up to 32 visits; reads stay inside the strip's list region)
  const int first_id = lane < re - rs ? __ldg(vl + 1 + lane) : -1;
  if (cnt < 0 || cnt > re - rs) {  // not a list the forward wrote for this strip
    if (lane == 0 && A.status) atomicExch(A.status, CS_ERR_ARG);
    return true;
  }
  ++vl;
  const long long wslot = visit_base(g) + 1;  // visit-list slot of position 0
  const DEntry* dl = A.dl + g.base;
  int q = cnt - 1;      // next position (walking down)
  int qb = cnt;         // first position of the batch in shared memory
  unsigned amask = 0u;  // active intersects of the batch
  int pf = -1;          // position whose winning records are in slot `slot`
  int slot = 0;
  while (q >= 0) {
    if (q < qb) {
      qb = max(0, q - 31);
      __syncwarp();  // every lane is done with the previous batch's codes
      stage_codes(A.winners + (wslot + qb) * 32, q - qb + 1, db);
      amask = load_batch<false>(A, vl + qb, rs + qb, q - qb + 1, st, rs, re, ib, qb == 0,
                                first_id);
      cp_async_wait_all();
      __syncwarp();  // the codes are visible to every lane
    }
    const int j = q - qb;
    if (!((amask >> j) & 1u)) {  // skip to the batch's next lower active intersect
      const unsigned below = amask & ((1u << j) - 1u);
      q = below ? qb + 31 - __clz(below) : qb - 1;
      continue;
    }
    if (pf != q) {  // the first visit of a batch
      slot ^= 1;
      prefetch_winners(dl, ib, j, s, db, slot);
    }
    const int k = ib.kk[j];
    const bool v0 = s[0].in && k <= s[0].fidx;
    const bool v1 = s[1].in && k <= s[1].fidx;
    IMeta m;
    batch_meta(ib, j, m);
    const int2 rg = ib.rg[j];
    const int ds = rg.x, nrec = rg.y;
    const unsigned wc = db.codes[j * 32 + lane];
    cp_async_wait_all();  // this visit's winning records
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const unsigned c = (wc >> (8 * u)) & 255u;
      const int win = (int)(c & 127u);
      s[u].w = s[u].n = (int)(c >> 7);
      s[u].md = 1e30f;
      s[u].be = -1;
      s[u].bl = -1;
      s[u].bp = s[u].bcx = s[u].bcy = 0.0f;
      if (nrec <= 0 || !(u ? v1 : v0)) continue;
      float4 EA, EB;
      if (win == kNoWinner) {  // walk the intersect's records (strict <: first minimum)
        int d = -1;
        for (int e = ds; e < ds + nrec; ++e) {
          const float4 WA = __ldg(&dl[e].a), WB = __ldg(&dl[e].b);
          float pr, cx, cy;
          const float d2 = seg_d2(px[u], py, py - WA.y, WA, WB, pr, cx, cy);
          if (d2 < s[u].md) {
            s[u].md = d2;
            d = e;
          }
        }
        if (d < 0) continue;
        EA = __ldg(&dl[d].a);
        EB = __ldg(&dl[d].b);
      } else if (win >= nrec) {  // not a code the forward wrote for this intersect
        if (A.status) atomicExch(A.status, CS_ERR_ARG);
        continue;
      } else {
        EA = db.ra[slot][u][lane];
        EB = db.rb[slot][u][lane];
      }
      s[u].md = seg_d2(px[u], py, py - EA.y, EA, EB, s[u].bp, s[u].bcx, s[u].bcy);
      s[u].be = __float_as_int(EB.w);
    }
    // the next active visit of the batch: its records load while this one computes
    {
      const unsigned below = amask & ((1u << j) - 1u);
      pf = -1;
      if (below) {
        const int jn = 31 - __clz(below);
        slot ^= 1;  // the other slot: this visit's records stay untouched
        prefetch_winners(dl, ib, jn, s, db, slot);
        pf = qb + jn;
      }
    }
    float acc[kAcc];
#pragma unroll
    for (int a = 0; a < kAcc; ++a) acc[a] = 0.0f;
    bool contributed = false;
    float4 eg[2];
    bool has_eg[2];
#pragma unroll
    for (int u = 0; u < 2; ++u)
      bwd_pixel<false>(s[u], m, px[u], py, u ? v1 : v0, acc, collect, A.v_opac != nullptr,
                       A.v_inv != nullptr, eg[u], has_eg[u], contributed);
    const bool any_c = __any_sync(0xffffffffu, contributed);
    const float a4[4] = {acc[0], acc[1], acc[2], A.v_opac ? acc[3] : 0.0f};
    const bool folded = add_edge_grads_direct(A, -(s[0].be + 2), has_eg[0], eg[0],
                                              -(s[1].be + 2), has_eg[1], eg[1],
                                              any_c && !A.v_inv && !collect, a4, m.pid, k);
    if (any_c && !folded) {
      const int vi = (lane >> 3) & 3;
      const bool leader = (lane & 7) == 0;
      float r = warp_reduce4(acc[0], acc[1], acc[2], A.v_opac ? acc[3] : 0.0f);
      if (leader) flush_acc(A, m.pid, k, vi, r);
      if (A.v_inv) {
        r = warp_reduce4(acc[4], 0.0f, 0.0f, 0.0f);
        if (leader && vi == 0) flush_acc(A, m.pid, k, 4, r);
      }
      if (collect) {
        r = warp_reduce4(acc[6], acc[7], acc[8], acc[9]);
        if (leader) flush_acc(A, m.pid, k, 6 + vi, r);
      }
    }
    --q;
  }
  cp_async_wait_all();  // nothing in flight into the buffers of the next unit
  return true;
}

// The fill backward over visit lists and winner codes (backward_unit_direct):
// no record staging, so no record buffers or mbarriers.
__global__ void __launch_bounds__(kRT) raster_backward_direct_kernel(const RasterArgs A) {
  __shared__ __align__(16) IBatch sib[kRW];
  __shared__ __align__(16) DirectBuf sdb[kRW];
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int pre0 = 0, pre1 = 0;
  if (A.order) unit_prefix(A.order, pre0, pre1);
  int u = blockIdx.x * kRW + wid;
  while (u < A.nunits) {
    const int unit = A.order ? unit_at(A.order, A.nunits, u, pre0, pre1) : u;
    if ((unsigned)unit >= (unsigned)A.nunits) {  // malformed dispatch lists
      if (lane == 0 && A.status) atomicExch(A.status, CS_ERR_ARG);
      break;
    }
    backward_unit_direct(A, unit, sib[wid], sdb[wid]);
    u = next_unit(A);
  }
  finish_launch(A, false);
}

template <bool STROKE>
__global__ void __launch_bounds__(kRT) raster_backward_kernel(const RasterArgs A) {
  __shared__ __align__(128) DEntry sbuf[kRW][2][kWChunk];
  __shared__ __align__(16) float4 sgrad[kRW][kWChunk];
  __shared__ __align__(16) IBatch sib[kRW];
  __shared__ __align__(8) uint64_t sbar[kRW][2];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint64_t* bars = sbar[wid];
  float4* dgrad = sgrad[wid];
  for (int q = lane; q < kWChunk; q += 32) dgrad[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane == 0) {
    mbar_init(&bars[0]);
    mbar_init(&bars[1]);
    fence_barrier_init();
  }
  __syncwarp();
  uint32_t phase = 0u;
  int pre0 = 0, pre1 = 0;
  if (A.order) unit_prefix(A.order, pre0, pre1);
  int u = blockIdx.x * kRW + wid;
  while (u < A.nunits) {
    const int unit = A.order ? unit_at(A.order, A.nunits, u, pre0, pre1) : u;
    if ((unsigned)unit >= (unsigned)A.nunits) {  // malformed dispatch lists
      if (lane == 0 && A.status) atomicExch(A.status, CS_ERR_ARG);
      break;
    }
    if (!backward_unit<STROKE>(A, unit, sbuf[wid], bars, phase, dgrad, sib[wid])) break;
    u = next_unit(A);
  }
  finish_launch(A, false);
}

// ---------------------------------------------------------------------------
// host launch

// Persistent grid: as many CTAs as fit on the device at once (cached per
// kernel and device), no more than the units need.  ID tells the kernels
// apart (they share one function type).
template <int ID, typename K>
inline int persistent_ctas(K kernel, int nunits) {
  constexpr int kMaxDev = 64;
  static int sms[kMaxDev] = {0};
  static int occ[kMaxDev] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) dev = 0;
  if (sms[dev] == 0) {
    int n = 0, o = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kernel, kRT, 0);
    occ[dev] = max(1, o);
    sms[dev] = max(1, n);
  }
  const int need = (nunits + kRW - 1) / kRW;
  return max(1, min(need, sms[dev] * occ[dev]));
}

inline int launch_raster(bool stroke, bool bwd, const RasterArgs& a, int H, int W, int r_begin,
                         int r_end, cudaStream_t st) {
  const int tbx = (W + kTile - 1) / kTile, tby = (H + kTile - 1) / kTile;
  const int r0 = max(0, r_begin), r1 = min(tby, r_end);
  if (r1 <= r0) return CS_OK;
  RasterArgs args = a;
  args.tbx = tbx;
  args.r0 = r0;
  args.H = H;
  args.W = W;
  args.nunits = kStrips * tbx * (r1 - r0);
  {
    auto al8 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 7u) == 0; };
    args.vec2 = (W % 2 == 0) && al8(args.fts) && al8(args.fidx) && al8(args.out) &&
                al8(args.out_chw) && al8(args.loss_tgt) && al8(args.fts_in) &&
                al8(args.fidx_in) && al8(args.v_out) && al8(args.out_img) && al8(args.tgt);
  }
  if (!stroke && !bwd) {
    auto k = raster_forward_kernel<false>;
    k<<<persistent_ctas<0>(k, args.nunits), kRT, 0, st>>>(args);
  } else if (stroke && !bwd) {
    auto k = raster_forward_kernel<true>;
    k<<<persistent_ctas<1>(k, args.nunits), kRT, 0, st>>>(args);
  } else if (!stroke && bwd && args.visits && args.winners &&
             ((reinterpret_cast<uintptr_t>(args.winners) |
               reinterpret_cast<uintptr_t>(args.dl)) & 15u) == 0) {
    // (the direct kernel copies codes and records 16 bytes at a time)
    auto k = raster_backward_direct_kernel;
    k<<<persistent_ctas<4>(k, args.nunits), kRT, 0, st>>>(args);
  } else if (!stroke && bwd) {
    auto k = raster_backward_kernel<false>;
    k<<<persistent_ctas<2>(k, args.nunits), kRT, 0, st>>>(args);
  } else {
    auto k = raster_backward_kernel<true>;
    k<<<persistent_ctas<3>(k, args.nunits), kRT, 0, st>>>(args);
  }
  return launch_status();
}

inline void stage_args(RasterArgs& a, const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                       const int32_t* tile_dlist, const void* imeta, const int32_t* isect_strips,
                       const int32_t* rowoff, const void* dlist, const int32_t* unit_order,
                       const float* background, int32_t* status, void* workspace) {
  a.pids = prim_ids_sorted;
  a.bins = tile_bins;
  a.dlr = reinterpret_cast<const int2*>(tile_dlist);
  a.meta = reinterpret_cast<const IMeta*>(imeta);
  a.istrip = reinterpret_cast<const int2*>(isect_strips);
  a.rowoff = rowoff;
  a.dl = reinterpret_cast<const DEntry*>(dlist);
  a.order = unit_order;
  a.bg = background;
  a.status = status;
  char* w = static_cast<char*>(workspace);
  a.queue = reinterpret_cast<unsigned*>(w);
  a.ticket = reinterpret_cast<unsigned*>(w + 4);
  a.partials = reinterpret_cast<float*>(w + 256);
}

}  // namespace cs

using namespace cs;

extern "C" {

size_t cs_visit_winners_size(int64_t isect_capacity, int64_t num_tiles) {
  return 16 * cs_visit_lists_size(isect_capacity, num_tiles);  // 32 x 2 bytes per list slot
}

size_t cs_visit_lists_size(int64_t isect_capacity, int64_t num_tiles) {
  const int64_t n = (isect_capacity > 0 ? isect_capacity : 0) + (num_tiles > 0 ? num_tiles : 1);
  return sizeof(int32_t) * (size_t)kStrips * (size_t)n;
}

size_t cs_raster_workspace_size(int64_t num_tiles) {
  return 256 + sizeof(float) * (size_t)kStrips * (size_t)(num_tiles > 0 ? num_tiles : 1);
}

static int raster_forward(bool stroke, const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                          const int32_t* tile_dlist, const void* imeta,
                          const int32_t* isect_strips, const int32_t* rowoff, const void* dlist,
                          const int32_t* unit_order, int32_t* unit_order_bwd,
                          int32_t* visit_lists, uint16_t* visit_winners,
                          const float* background, float* out_img, float* final_Ts,
                          int32_t* final_idx, float* out_chw_clamped, const float* target_chw,
                          float* loss_out, int32_t* status, void* workspace, int32_t img_height,
                          int32_t img_width, int32_t tile_row_begin, int32_t tile_row_end,
                          void* stream) {
  if (img_height <= 0 || img_width <= 0 || !tile_bins || !tile_dlist || !imeta || !isect_strips ||
      !dlist || !background || !out_img || !final_Ts || !final_idx || !workspace ||
      (!stroke && !rowoff) || (target_chw && !loss_out))
    return CS_ERR_ARG;
  RasterArgs a{};
  stage_args(a, prim_ids_sorted, tile_bins, tile_dlist, imeta, isect_strips, rowoff, dlist,
             unit_order, background, status, workspace);
  a.order_next = unit_order_bwd;
  a.visits = visit_lists;
  a.winners = visit_lists ? visit_winners : nullptr;
  if (unit_order_bwd)
    cudaMemsetAsync(unit_order_bwd, 0, sizeof(int32_t) * kUnitBuckets, (cudaStream_t)stream);
  a.out = out_img;
  a.fts = final_Ts;
  a.fidx = final_idx;
  a.out_chw = out_chw_clamped;
  a.loss_tgt = target_chw;
  a.loss_out = loss_out;
  return launch_raster(stroke, false, a, img_height, img_width, tile_row_begin, tile_row_end,
                       (cudaStream_t)stream);
}

int cs_fill_forward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                    const int32_t* tile_dlist, const void* imeta, const int32_t* isect_strips,
                    const int32_t* rowoff, const void* dlist, const int32_t* unit_order,
                    int32_t* unit_order_bwd, int32_t* visit_lists, uint16_t* visit_winners,
                    const float* background, float* out_img, float* final_Ts,
                    int32_t* final_idx, float* out_chw_clamped, const float* target_chw,
                    float* loss_out, int32_t* status, void* workspace, int32_t img_height,
                    int32_t img_width, int32_t tile_row_begin, int32_t tile_row_end,
                    void* stream) {
  return raster_forward(false, prim_ids_sorted, tile_bins, tile_dlist, imeta, isect_strips,
                        rowoff, dlist, unit_order, unit_order_bwd, visit_lists, visit_winners,
                        background, out_img, final_Ts, final_idx,
                        out_chw_clamped, target_chw, loss_out, status, workspace, img_height,
                        img_width, tile_row_begin, tile_row_end, stream);
}

int cs_stroke_forward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                      const int32_t* tile_dlist, const void* imeta, const int32_t* isect_strips,
                      const void* dlist, const int32_t* unit_order, int32_t* unit_order_bwd,
                      int32_t* visit_lists, uint16_t* visit_winners, const float* background,
                      float* out_img, float* final_Ts, int32_t* final_idx,
                      float* out_chw_clamped, const float* target_chw, float* loss_out,
                      int32_t* status, void* workspace, int32_t img_height, int32_t img_width,
                      int32_t tile_row_begin, int32_t tile_row_end, void* stream) {
  return raster_forward(true, prim_ids_sorted, tile_bins, tile_dlist, imeta, isect_strips,
                        nullptr, dlist, unit_order, unit_order_bwd, visit_lists, visit_winners,
                        background, out_img, final_Ts, final_idx,
                        out_chw_clamped, target_chw, loss_out, status, workspace, img_height,
                        img_width, tile_row_begin, tile_row_end, stream);
}

static int raster_backward(bool stroke, const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                           const int32_t* tile_dlist, const void* imeta,
                           const int32_t* isect_strips, const int32_t* rowoff, const void* dlist,
                           const int32_t* unit_order, const int32_t* visit_lists,
                           const uint16_t* visit_winners, const float* background,
                           const float* final_Ts,
                           const int32_t* final_idx,
                           const float* v_output, const float* out_img, const float* target_chw,
                           const float* mse_scale, float* v_edges, float* v_colors,
                           float* v_opacities, float* v_stroke_widths, float* v_inv_sigma2s,
                           float* curve_contrib_rgb, float* curve_isect_contrib,
                           int32_t* status, void* workspace, int32_t img_height,
                           int32_t img_width, int32_t tile_row_begin, int32_t tile_row_end,
                           void* stream) {
  if (img_height <= 0 || img_width <= 0 || !prim_ids_sorted || !tile_bins || !tile_dlist ||
      !imeta || !isect_strips || !dlist || !background || !final_Ts || !final_idx || !v_edges ||
      !v_colors || !workspace || (!stroke && !rowoff) || (stroke && !v_stroke_widths))
    return CS_ERR_ARG;
  if (!v_output && (!out_img || !target_chw || !mse_scale)) return CS_ERR_ARG;
  RasterArgs a{};
  stage_args(a, prim_ids_sorted, tile_bins, tile_dlist, imeta, isect_strips, rowoff, dlist,
             unit_order, background, status, workspace);
  a.visits = const_cast<int32_t*>(visit_lists);  // read only by the backward
  a.winners = visit_lists ? const_cast<uint16_t*>(visit_winners) : nullptr;
  a.fts_in = final_Ts;
  a.fidx_in = final_idx;
  a.v_out = v_output;
  a.out_img = out_img;
  a.tgt = target_chw;
  a.mse_scale = mse_scale;
  a.v_edges = v_edges;
  a.v_colors = v_colors;
  a.v_opac = v_opacities;
  a.v_sw = v_stroke_widths;
  a.v_inv = v_inv_sigma2s;
  a.contrib = curve_contrib_rgb;
  a.icontrib = curve_isect_contrib;
  return launch_raster(stroke, true, a, img_height, img_width, tile_row_begin, tile_row_end,
                       (cudaStream_t)stream);
}

int cs_fill_backward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                     const int32_t* tile_dlist, const void* imeta, const int32_t* isect_strips,
                     const int32_t* rowoff, const void* dlist, const int32_t* unit_order,
                     const int32_t* visit_lists, const uint16_t* visit_winners,
                     const float* background, const float* final_Ts, const int32_t* final_idx,
                     const float* v_output, const float* out_img, const float* target_chw,
                     const float* mse_scale, float* v_edges, float* v_colors,
                     float* v_opacities, float* v_inv_sigma2s, float* curve_contrib_rgb,
                     float* curve_isect_contrib, int32_t* status, void* workspace,
                     int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                     int32_t tile_row_end, void* stream) {
  return raster_backward(false, prim_ids_sorted, tile_bins, tile_dlist, imeta, isect_strips,
                         rowoff, dlist, unit_order, visit_lists, visit_winners, background, final_Ts,
                         final_idx,
                         v_output,
                         out_img, target_chw, mse_scale, v_edges, v_colors, v_opacities, nullptr,
                         v_inv_sigma2s, curve_contrib_rgb, curve_isect_contrib, status,
                         workspace, img_height, img_width, tile_row_begin, tile_row_end, stream);
}

int cs_stroke_backward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                       const int32_t* tile_dlist, const void* imeta, const int32_t* isect_strips,
                       const void* dlist, const int32_t* unit_order,
                       const int32_t* visit_lists, const uint16_t* visit_winners,
                       const float* background, const float* final_Ts, const int32_t* final_idx,
                       const float* v_output,
                       const float* out_img, const float* target_chw, const float* mse_scale,
                       float* v_edges, float* v_colors, float* v_opacities,
                       float* v_stroke_widths, float* v_inv_sigma2s, float* curve_contrib_rgb,
                       float* curve_isect_contrib, int32_t* status, void* workspace,
                       int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                       int32_t tile_row_end, void* stream) {
  return raster_backward(true, prim_ids_sorted, tile_bins, tile_dlist, imeta, isect_strips,
                         nullptr, dlist, unit_order, visit_lists, visit_winners, background, final_Ts,
                         final_idx,
                         v_output,
                         out_img, target_chw, mse_scale, v_edges, v_colors, v_opacities,
                         v_stroke_widths, v_inv_sigma2s, curve_contrib_rgb, curve_isect_contrib,
                         status, workspace, img_height, img_width, tile_row_begin, tile_row_end,
                         stream);
}

}  // extern "C"
