// Per-tile rasterisation of closed fills and open strokes, forward and
// backward (sm_100a).
//
// One CTA per 16x16 tile, 128 threads, two horizontally adjacent pixels per
// thread.  The tile's intersects (front-to-back in the forward, back-to-front
// in the backward) are staged in batches: warp 0 gathers up to 32 intersects
// ("pieces"; a primitive with more than kDCap edges is split into several
// pieces) and the CTA classifies every edge of the batch against the tile:
//
//  * near edges -- the edge's bounding box comes within d_thr of the tile's
//    pixel-centre box -- are compacted, in edge order, into a shared-memory
//    list with their per-frame constants (direction, 1/|d|^2, x0*dy);
//  * far edges whose y-span crosses tile rows and that lie entirely to the
//    right of the tile add +-1 to per-row winding offsets (every pixel of such
//    a row is crossed by them, far beyond rounding error);
//  * all other edges cannot touch any pixel of the tile and are dropped.
//
// d_thr is the distance beyond which a pixel's coverage is saturated for the
// primitive: fill coverage is exactly 1.0f inside (logit <= -20) and below
// alpha_min outside; stroke coverage is below alpha_min.  A pixel closer than
// d_thr to the polyline has its closest edge in the near list, so its
// distance is the exact minimum; a farther pixel gets a saturated coverage
// whichever edges are visited.  Results are therefore those of visiting every
// edge, which is what the reference does
// (manbo/ops/cubic_splatting.py:1070-1136 and :1429-1501).
//
// Per-pixel arithmetic follows the reference formulas in their written order
// (-fmad=false); exp is cs_expf.  The backward recomputes the geometry with
// the first-minimum closest edge (lexicographic on (d^2, edge id)), walks the
// intersects in reverse with T <- T / (1 - alpha), reduces per-primitive
// gradients over the warp and the CTA in shared memory, and accumulates edge
// gradients per near edge in shared memory before one global atomic per edge.
#include <math_constants.h>

#include "cs_common.cuh"

namespace cs {

constexpr int kRT = 128;     // threads per CTA: 16 rows x 8 pixel pairs
constexpr int kDCap = 512;   // near-edge entries per batch (4 edges per thread)
constexpr int kNP = 32;      // pieces per batch (one per lane of warp 0)
constexpr int kFirst = 1;    // piece holds the first edge of its intersect
constexpr int kLast = 2;     // piece holds the last edge of its intersect
constexpr int kAcc = 10;     // per-piece gradient accumulators

struct __align__(16) Piece {
  int k, pid, ebeg, eend;
  int flat, dstart, dcount, flags;
  float c0, c1, c2, op;
  float a;     // fill: inv_sigma = sqrt(max(inv_sigma2, eps)); stroke: max(inv_sigma2, eps)
  float b;     // stroke: half stroke width
  float dthr;  // culling distance
  int rule;    // fill rule (0 even-odd, else nonzero)
};

template <bool BWD>
struct Smem {
  Piece piece[kNP];
  float4 dA[kDCap];  // x0, y0, vx, vy
  float4 dB[kDCap];  // 1/max(|v|^2, eps), y1, x0*vy, edge id (bits)
  int rowwind[kNP][16];
  int rowcnt[kNP][16];
  int pcount[kNP];
  int warp_tot[kRT / 32];
  int npieces, total, ndl;
  int next_k, next_e;
  float pacc[BWD ? kNP : 1][kAcc];
  float4 dgrad[BWD ? kDCap : 1];
};

struct RasterArgs {
  const int* pids;
  const int* bins;
  const float4* edges;
  const int2* ranges;
  const int* eoffs;
  const float* colors;
  const float* opac;
  const float* inv_s2;
  const int* rules;
  const float* sw;
  const float* bg;
  int H, W, tbx, r0;
  // forward outputs
  float* out;
  float* fts;
  int* fidx;
  float* out_chw;  // optional clamp(out, 0, 1) in [3, H, W]
  // backward inputs / outputs
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

// ---------------------------------------------------------------------------
// batch construction (warp 0)

template <bool STROKE>
__device__ __forceinline__ void fill_piece_attrs(Piece& pc, const RasterArgs& A) {
  const int pid = pc.pid;
  pc.c0 = A.colors[pid * 3];
  pc.c1 = A.colors[pid * 3 + 1];
  pc.c2 = A.colors[pid * 3 + 2];
  const float op = A.opac[pid];
  pc.op = op;
  const float is2 = A.inv_s2[pid];
  const float lg = logf(fmaxf(255.0f * op, 1.0f)) + 1.0f;
  if (!STROKE) {
    pc.a = sqrtf(fmaxf(is2, kEps));
    pc.b = 0.0f;
    pc.rule = A.rules[pid];
    const float L = fmaxf(20.0f, lg);
    pc.dthr = (L <= 59.0f && pc.a > 0.0f) ? 0.5f * L / pc.a + 0.5f : CUDART_INF_F;
  } else {
    pc.a = fmaxf(is2, kEps);
    pc.b = fmaxf(0.0f, A.sw[pid]) * 0.5f;
    pc.rule = 1;
    pc.dthr = pc.b + sqrtf(2.0f * lg / pc.a) + 0.5f;
  }
  if (!(pc.dthr == pc.dthr)) pc.dthr = CUDART_INF_F;
}

// Fills piece[0..npieces) for the next batch.  Forward (REV = false) walks
// intersects upward from next_k; next_e counts edges of next_k already
// consumed.  Backward walks downward; next_e is the absolute end of the edges
// of next_k still to visit (-1 = all).  Sets npieces = 0 when done.
template <bool STROKE, bool REV, bool BWD>
__device__ void build_batch(Smem<BWD>& sm, const RasterArgs& A, int rs, int re, int lane) {
  const int nk = sm.next_k, ne = sm.next_e;
  const int k = REV ? nk - lane : nk + lane;
  const bool valid = REV ? (k >= rs) : (k < re);
  int pid = 0, eb = 0, ee = 0;
  if (valid) {
    pid = A.pids[k];
    if (A.ranges) {
      int2 r = A.ranges[k];
      eb = r.x;
      ee = r.y;
    } else {
      eb = A.eoffs[pid];
      ee = A.eoffs[pid + 1];
    }
    if (!REV && lane == 0) eb += ne;
    if (REV && lane == 0 && ne >= 0) ee = ne;
  }
  const int n = valid ? max(0, ee - eb) : 0;
  const int incl = warp_incl_scan(n, lane);
  const unsigned vmask = __ballot_sync(0xffffffffu, valid);
  const unsigned fmask = __ballot_sync(0xffffffffu, valid && incl <= kDCap);
  const int nvalid = __popc(vmask);
  const int cnt = __popc(fmask);
  __syncwarp();
  if (nvalid == 0) {
    if (lane == 0) sm.npieces = 0;
    return;
  }
  if (cnt == 0) {
    // The first intersect alone exceeds the staging capacity: one piece.
    if (lane == 0) {
      Piece pc;
      pc.k = k;
      pc.pid = pid;
      pc.flat = 0;
      if (!REV) {
        pc.ebeg = eb;
        pc.eend = eb + kDCap;
        pc.flags = (ne == 0) ? kFirst : 0;
        sm.next_e = ne + kDCap;
      } else {
        pc.eend = ee;
        pc.ebeg = ee - kDCap;
        pc.flags = (ne < 0) ? kLast : 0;
        sm.next_e = pc.ebeg;
      }
      fill_piece_attrs<STROKE>(pc, A);
      sm.piece[0] = pc;
      sm.npieces = 1;
      sm.total = kDCap;
    }
    return;
  }
  if (lane < cnt) {
    Piece pc;
    pc.k = k;
    pc.pid = pid;
    pc.ebeg = eb;
    pc.eend = ee;
    pc.flat = incl - n;
    if (!REV)
      pc.flags = kLast | ((lane > 0 || ne == 0) ? kFirst : 0);
    else
      pc.flags = kFirst | ((lane > 0 || ne < 0) ? kLast : 0);
    fill_piece_attrs<STROKE>(pc, A);
    sm.piece[lane] = pc;
  }
  if (lane == cnt - 1) {
    sm.npieces = cnt;
    sm.total = incl;
    sm.next_k = REV ? nk - cnt : nk + cnt;
    sm.next_e = REV ? -1 : 0;
  }
}

// ---------------------------------------------------------------------------
// edge classification and near-list compaction (all threads)

template <bool STROKE, bool BWD>
__device__ void stage_batch(Smem<BWD>& sm, const RasterArgs& A, int tx, int ty, int tid) {
  const int lane = tid & 31, wid = tid >> 5;
  const int tot = sm.total, np = sm.npieces;
  const float bx0 = (float)(tx * kTile) + 0.5f, bx1 = bx0 + 15.0f;
  const float by0 = (float)(ty * kTile) + 0.5f, by1 = by0 + 15.0f;
  const int q0 = tid * 4;
  float4 ev[4];
  int eidv[4];
  unsigned nearbits = 0;
  int mycount = 0;
  if (q0 < tot) {
    // piece containing q0: last piece whose flat <= q0
    int lo = 0, hi = np - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (sm.piece[mid].flat <= q0) lo = mid; else hi = mid - 1;
    }
    int pc = lo;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = q0 + u;
      if (q >= tot) break;
      while (pc + 1 < np && sm.piece[pc + 1].flat <= q) ++pc;
      const Piece& P = sm.piece[pc];
      const int eid = P.ebeg + (q - P.flat);
      const float4 e = A.edges[eid];
      ev[u] = e;
      eidv[u] = eid;
      const float d = P.dthr;
      const float xmin = fminf(e.x, e.z), xmax = fmaxf(e.x, e.z);
      const float ymin = fminf(e.y, e.w), ymax = fmaxf(e.y, e.w);
      const bool moderate = fabsf(e.x) < 4.0e6f && fabsf(e.y) < 4.0e6f && fabsf(e.z) < 4.0e6f &&
                            fabsf(e.w) < 4.0e6f;
      const bool near = !moderate || (xmax >= bx0 - d && xmin <= bx1 + d && ymax >= by0 - d &&
                                      ymin <= by1 + d);
      if (near) {
        nearbits |= 1u << u;
        ++mycount;
        atomicAdd(&sm.pcount[pc], 1);
      } else if (!STROKE && xmin > bx1 && ymax >= by0 && ymin <= by1) {
        // entirely right of the tile: crosses every pixel of the rows it spans
        const float vy = e.w - e.y;
        const int dir = vy > 0.0f ? 1 : -1;
#pragma unroll 4
        for (int r = 0; r < 16; ++r) {
          const float py = by0 + (float)r;
          if (((e.y <= py) & (e.w > py)) | ((e.y > py) & (e.w <= py))) {
            atomicAdd(&sm.rowwind[pc][r], dir);
            atomicAdd(&sm.rowcnt[pc][r], 1);
          }
        }
      }
    }
  }
  // block exclusive scan of the per-thread near counts (edge order preserved)
  const int incl = warp_incl_scan(mycount, lane);
  if (lane == 31) sm.warp_tot[wid] = incl;
  __syncthreads();
  int base = 0;
#pragma unroll
  for (int w = 0; w < kRT / 32; ++w) base += (w < wid) ? sm.warp_tot[w] : 0;
  int pos = base + incl - mycount;
  if (tid == kRT - 1) sm.ndl = base + incl;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (nearbits & (1u << u)) {
      const float4 e = ev[u];
      const float vx = e.z - e.x, vy = e.w - e.y;
      const float vv = vx * vx + vy * vy;
      const float inv_vv = 1.0f / fmaxf(vv, kEps);
      sm.dA[pos] = make_float4(e.x, e.y, vx, vy);
      sm.dB[pos] = make_float4(inv_vv, e.w, e.x * vy, __int_as_float(eidv[u]));
      ++pos;
    }
  }
  if (wid == 0) {
    const int c = lane < np ? sm.pcount[lane] : 0;
    const int ci = warp_incl_scan(c, lane);
    if (lane < np) {
      sm.piece[lane].dstart = ci - c;
      sm.piece[lane].dcount = c;
    }
  }
}

template <bool BWD>
__device__ __forceinline__ void zero_batch_smem(Smem<BWD>& sm, int tid) {
  int* rw = &sm.rowwind[0][0];
  int* rc = &sm.rowcnt[0][0];
  for (int i = tid; i < kNP * 16; i += kRT) {
    rw[i] = 0;
    rc[i] = 0;
  }
  if (tid < kNP) sm.pcount[tid] = 0;
  if (BWD) {
    float* pa = &sm.pacc[0][0];
    for (int i = tid; i < kNP * kAcc; i += kRT) pa[i] = 0.0f;
    for (int i = tid; i < kDCap; i += kRT) sm.dgrad[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// ---------------------------------------------------------------------------
// per-pixel geometry

struct FwdGeom {
  float md;
  int w, n;
};

__device__ __forceinline__ float seg_d2(float px, float py, float wy, const float4& A,
                                        const float4& B, float& proj, float& cx, float& cy) {
  const float wx = px - A.x;
  float pr = (wx * A.z + wy * A.w) * B.x;
  pr = fmaxf(0.0f, fminf(1.0f, pr));
  cx = A.x + pr * A.z;
  cy = A.y + pr * A.w;
  const float dx = cx - px, dy = cy - py;
  proj = pr;
  return dx * dx + dy * dy;
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

// ---------------------------------------------------------------------------
// forward

template <bool STROKE>
__global__ void __launch_bounds__(kRT) raster_forward_kernel(const RasterArgs A) {
  __shared__ Smem<false> sm;
  const int tid = threadIdx.x, lane = tid & 31;
  const int tx = blockIdx.x, ty = A.r0 + blockIdx.y;
  const long long tile = (long long)ty * A.tbx + tx;
  const int rs = A.bins[2 * tile], re = A.bins[2 * tile + 1];
  const int ly = tid >> 3, lx = (tid & 7) * 2;
  const int i = ty * kTile + ly, j0 = tx * kTile + lx;
  const bool in0 = i < A.H && j0 < A.W, in1 = i < A.H && j0 + 1 < A.W;
  const float py = (float)i + 0.5f;
  const float px0 = (float)j0 + 0.5f, px1 = (float)(j0 + 1) + 0.5f;
  float T0 = 1.0f, T1 = 1.0f;
  float a00 = 0.f, a01 = 0.f, a02 = 0.f, a10 = 0.f, a11 = 0.f, a12 = 0.f;
  int cur0 = 0, cur1 = 0;
  bool d0 = !in0, d1 = !in1;
  FwdGeom g0{1e30f, 0, 0}, g1{1e30f, 0, 0};
  if (tid == 0) {
    sm.next_k = rs;
    sm.next_e = 0;
  }
  __syncthreads();
  while (true) {
    if (__syncthreads_count(!(d0 && d1)) == 0) break;
    zero_batch_smem<false>(sm, tid);
    if (tid < 32) build_batch<STROKE, false, false>(sm, A, rs, re, lane);
    __syncthreads();
    const int np = sm.npieces;
    if (np == 0) break;
    stage_batch<STROKE, false>(sm, A, tx, ty, tid);
    __syncthreads();
    for (int pc = 0; pc < np; ++pc) {
      const bool act = !(d0 && d1);
      if (!__any_sync(0xffffffffu, act)) continue;
      const Piece& P = sm.piece[pc];
      const int flags = P.flags, ds = P.dstart, de = P.dstart + P.dcount;
      if (flags & kFirst) {
        g0 = FwdGeom{1e30f, 0, 0};
        g1 = FwdGeom{1e30f, 0, 0};
      }
      for (int d = ds; d < de; ++d) {
        const float4 EA = sm.dA[d];
        const float4 EB = sm.dB[d];
        const float wy = py - EA.y;
        float pr, cx, cy;
        g0.md = fminf(g0.md, seg_d2(px0, py, wy, EA, EB, pr, cx, cy));
        g1.md = fminf(g1.md, seg_d2(px1, py, wy, EA, EB, pr, cx, cy));
        if (!STROKE) {
          if (((EA.y <= py) & (EB.y > py)) | ((EA.y > py) & (EB.y <= py))) {
            const float lhs = EB.z + wy * EA.z;
            const float rhs0 = px0 * EA.w, rhs1 = px1 * EA.w;
            const bool pos = EA.w > 0.0f;
            const int h0 = pos ? (lhs > rhs0) : (lhs < rhs0);
            const int h1 = pos ? (lhs > rhs1) : (lhs < rhs1);
            const int sg = pos ? 1 : -1;
            g0.n += h0;
            g1.n += h1;
            g0.w += h0 * sg;
            g1.w += h1 * sg;
          }
        }
      }
      if (!STROKE) {
        const int rw = sm.rowwind[pc][ly], rc = sm.rowcnt[pc][ly];
        g0.w += rw;
        g1.w += rw;
        g0.n += rc;
        g1.n += rc;
      }
      if (flags & kLast) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const bool dn = u ? d1 : d0;
          if (dn) continue;
          const FwdGeom& g = u ? g1 : g0;
          float cov;
          if (!STROKE) {
            float sign, dist;
            cov = fill_coverage(g.md, g.w, g.n, P.rule, P.a, sign, dist);
          } else {
            float dist, edge_d;
            cov = stroke_coverage(g.md, P.b, P.a, dist, edge_d);
          }
          const float alpha = fminf(kAlphaCap, P.op * cov);
          if (alpha < kAlphaMin) continue;
          float& T = u ? T1 : T0;
          const float nT = T * (1.0f - alpha);
          const float vis = alpha * T;
          if (u) {
            a10 += P.c0 * vis; a11 += P.c1 * vis; a12 += P.c2 * vis;
            cur1 = P.k;
            if (nT <= kTransStop) d1 = true;
          } else {
            a00 += P.c0 * vis; a01 += P.c1 * vis; a02 += P.c2 * vis;
            cur0 = P.k;
            if (nT <= kTransStop) d0 = true;
          }
          T = nT;
        }
      }
    }
  }
  const float bg0 = A.bg[0], bg1 = A.bg[1], bg2 = A.bg[2];
  const long long hw = (long long)A.H * A.W;
  if (in0) {
    const long long pix = (long long)i * A.W + j0;
    const float o0 = a00 + T0 * bg0, o1 = a01 + T0 * bg1, o2 = a02 + T0 * bg2;
    A.fts[pix] = T0;
    A.fidx[pix] = cur0;
    A.out[pix * 3] = o0;
    A.out[pix * 3 + 1] = o1;
    A.out[pix * 3 + 2] = o2;
    if (A.out_chw) {
      A.out_chw[pix] = fminf(fmaxf(o0, 0.0f), 1.0f);
      A.out_chw[hw + pix] = fminf(fmaxf(o1, 0.0f), 1.0f);
      A.out_chw[2 * hw + pix] = fminf(fmaxf(o2, 0.0f), 1.0f);
    }
  }
  if (in1) {
    const long long pix = (long long)i * A.W + j0 + 1;
    const float o0 = a10 + T1 * bg0, o1 = a11 + T1 * bg1, o2 = a12 + T1 * bg2;
    A.fts[pix] = T1;
    A.fidx[pix] = cur1;
    A.out[pix * 3] = o0;
    A.out[pix * 3 + 1] = o1;
    A.out[pix * 3 + 2] = o2;
    if (A.out_chw) {
      A.out_chw[pix] = fminf(fmaxf(o0, 0.0f), 1.0f);
      A.out_chw[hw + pix] = fminf(fmaxf(o1, 0.0f), 1.0f);
      A.out_chw[2 * hw + pix] = fminf(fmaxf(o2, 0.0f), 1.0f);
    }
  }
}

// ---------------------------------------------------------------------------
// backward

struct BwdPix {
  float T, Tf, b0, b1, b2, v0, v1, v2, bgd;
  int fidx;
  bool in;
  // geometry of the current intersect
  float md, bp, bcx, bcy;
  int be, bl, w, n;
};

template <bool STROKE>
__device__ __forceinline__ void bwd_pixel(BwdPix& s, const Piece& P, float px, float py, bool valid,
                                          float acc[kAcc], bool collect, float4& eg, int& eg_loc,
                                          int& eg_eid, bool& contributed) {
  eg_loc = -1;
  eg_eid = -1;
  if (!valid) return;
  float cov, sign = 1.0f, dist, edge_d = 0.0f;
  if (!STROKE) {
    cov = fill_coverage(s.md, s.w, s.n, P.rule, P.a, sign, dist);
  } else {
    cov = stroke_coverage(s.md, P.b, P.a, dist, edge_d);
  }
  const float op = P.op;
  const float alpha = fminf(kAlphaCap, op * cov);
  if (!(alpha >= kAlphaMin)) return;
  contributed = true;
  const float ra = 1.0f / (1.0f - alpha);
  s.T = s.T * ra;
  const float fac = alpha * s.T;
  acc[0] += fac * s.v0;
  acc[1] += fac * s.v1;
  acc[2] += fac * s.v2;
  if (collect) {
    const float c0 = fac * P.c0, c1 = fac * P.c1, c2 = fac * P.c2;
    acc[6] += c0;
    acc[7] += c1;
    acc[8] += c2;
    acc[9] += c0 + c1 + c2;
  }
  float v_alpha = 0.0f;
  v_alpha = v_alpha + (P.c0 * s.T - s.b0 * ra) * s.v0;
  v_alpha = v_alpha + (P.c1 * s.T - s.b1 * ra) * s.v1;
  v_alpha = v_alpha + (P.c2 * s.T - s.b2 * ra) * s.v2;
  v_alpha = v_alpha + s.Tf * ra * (0.0f - s.bgd);
  s.b0 = s.b0 + P.c0 * fac;
  s.b1 = s.b1 + P.c1 * fac;
  s.b2 = s.b2 + P.c2 * fac;
  if (!(alpha < kAlphaCap)) return;
  acc[3] += cov * v_alpha;
  float gscale;  // d loss / d dist along (closest - pixel) / dist
  bool geom;
  if (!STROKE) {
    const float v_cov = op * v_alpha;
    const float v_logit = -v_cov * cov * (1.0f - cov);
    const float v_inv_sigma = v_logit * sign * dist * 2.0f;
    acc[4] += v_inv_sigma * 0.5f / fmaxf(P.a, kEps);
    gscale = v_logit * sign * P.a * 2.0f;
    geom = (dist > kEps) & (s.be >= 0);
  } else {
    const float v_sigma = -op * cov * v_alpha;
    acc[4] += 0.5f * edge_d * edge_d * v_sigma;
    geom = false;
    gscale = 0.0f;
    if (edge_d > 0.0f) {
      const float v_edge = v_sigma * edge_d * P.a;
      acc[5] += -0.5f * v_edge;
      gscale = v_edge;
      geom = (dist > kEps) & (s.be >= 0);
    }
  }
  if (geom) {
    const float gx = gscale * (s.bcx - px) / dist;
    const float gy = gscale * (s.bcy - py) / dist;
    eg = make_float4((1.0f - s.bp) * gx, (1.0f - s.bp) * gy, s.bp * gx, s.bp * gy);
    eg_loc = s.bl;
    eg_eid = s.be;
  }
}

template <bool STROKE>
__global__ void __launch_bounds__(kRT) raster_backward_kernel(const RasterArgs A) {
  __shared__ Smem<true> sm;
  const int tid = threadIdx.x, lane = tid & 31;
  const int tx = blockIdx.x, ty = A.r0 + blockIdx.y;
  const long long tile = (long long)ty * A.tbx + tx;
  const int rs = A.bins[2 * tile], re = A.bins[2 * tile + 1];
  if (re <= rs) return;
  const int ly = tid >> 3, lx = (tid & 7) * 2;
  const int i = ty * kTile + ly, j0 = tx * kTile + lx;
  const float py = (float)i + 0.5f;
  const float px[2] = {(float)j0 + 0.5f, (float)(j0 + 1) + 0.5f};
  const bool collect = (A.contrib != nullptr) | (A.icontrib != nullptr);
  const float scale = A.v_out ? 0.0f : *A.mse_scale;
  BwdPix s[2];
  int kmax = -1;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int j = j0 + u;
    s[u].in = i < A.H && j < A.W;
    s[u].b0 = s[u].b1 = s[u].b2 = 0.0f;
    s[u].md = 1e30f;
    s[u].be = -1;
    s[u].bl = -1;
    s[u].bp = s[u].bcx = s[u].bcy = 0.0f;
    s[u].w = s[u].n = 0;
    if (s[u].in) {
      const long long pix = (long long)i * A.W + j;
      s[u].T = A.fts_in[pix];
      s[u].fidx = A.fidx_in[pix];
      float v[3];
      if (A.v_out) {
        v[0] = A.v_out[pix * 3];
        v[1] = A.v_out[pix * 3 + 1];
        v[2] = A.v_out[pix * 3 + 2];
      } else {
        const long long hw = (long long)A.H * A.W;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          const float o = A.out_img[pix * 3 + c];
          const float t = A.tgt[c * hw + pix];
          v[c] = (o >= 0.0f && o <= 1.0f) ? scale * (o - t) : 0.0f;
        }
      }
      s[u].v0 = v[0];
      s[u].v1 = v[1];
      s[u].v2 = v[2];
      s[u].bgd = A.bg[0] * v[0] + A.bg[1] * v[1] + A.bg[2] * v[2];
      kmax = max(kmax, s[u].fidx);
    } else {
      s[u].T = 1.0f;
      s[u].fidx = -1;
      s[u].v0 = s[u].v1 = s[u].v2 = s[u].bgd = 0.0f;
    }
    s[u].Tf = s[u].T;
  }
  // highest intersect any pixel of the tile needs
  kmax = warp_max_i(kmax);
  if (lane == 0) sm.warp_tot[tid >> 5] = kmax;
  __syncthreads();
  if (tid == 0) {
    int m = sm.warp_tot[0];
    for (int w = 1; w < kRT / 32; ++w) m = max(m, sm.warp_tot[w]);
    sm.next_k = min(m, re - 1);
    sm.next_e = -1;
  }
  __syncthreads();
  if (sm.next_k < rs) return;
  while (true) {
    zero_batch_smem<true>(sm, tid);
    if (tid < 32) build_batch<STROKE, true, true>(sm, A, rs, re, lane);
    __syncthreads();
    const int np = sm.npieces;
    if (np == 0) break;
    stage_batch<STROKE, true>(sm, A, tx, ty, tid);
    __syncthreads();
    s[0].bl = -1;  // near lists are rebuilt every batch
    s[1].bl = -1;
    for (int pc = 0; pc < np; ++pc) {
      const Piece& P = sm.piece[pc];
      const bool v0 = s[0].in && P.k <= s[0].fidx;
      const bool v1 = s[1].in && P.k <= s[1].fidx;
      if (!__any_sync(0xffffffffu, v0 || v1)) continue;
      const int flags = P.flags, ds = P.dstart, de = P.dstart + P.dcount;
      if (flags & kLast) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          s[u].md = 1e30f;
          s[u].be = -1;
          s[u].bl = -1;
          s[u].bp = s[u].bcx = s[u].bcy = 0.0f;
          s[u].w = s[u].n = 0;
        }
      }
      for (int d = ds; d < de; ++d) {
        const float4 EA = sm.dA[d];
        const float4 EB = sm.dB[d];
        const int eid = __float_as_int(EB.w);
        const float wy = py - EA.y;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float pr, cx, cy;
          const float d2 = seg_d2(px[u], py, wy, EA, EB, pr, cx, cy);
          if (d2 < s[u].md || (d2 == s[u].md && eid < s[u].be)) {
            s[u].md = d2;
            s[u].be = eid;
            s[u].bl = d;
            s[u].bp = pr;
            s[u].bcx = cx;
            s[u].bcy = cy;
          }
        }
        if (!STROKE) {
          if (((EA.y <= py) & (EB.y > py)) | ((EA.y > py) & (EB.y <= py))) {
            const float lhs = EB.z + wy * EA.z;
            const bool pos = EA.w > 0.0f;
            const int sg = pos ? 1 : -1;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float rhs = px[u] * EA.w;
              const int h = pos ? (lhs > rhs) : (lhs < rhs);
              s[u].n += h;
              s[u].w += h * sg;
            }
          }
        }
      }
      if (!STROKE) {
        const int rw = sm.rowwind[pc][ly], rc = sm.rowcnt[pc][ly];
        s[0].w += rw;
        s[1].w += rw;
        s[0].n += rc;
        s[1].n += rc;
      }
      if (!(flags & kFirst)) continue;
      float acc[kAcc];
#pragma unroll
      for (int c = 0; c < kAcc; ++c) acc[c] = 0.0f;
      bool contributed = false;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float4 eg;
        int eg_loc, eg_eid;
        bwd_pixel<STROKE>(s[u], P, px[u], py, u ? v1 : v0, acc, collect, eg, eg_loc, eg_eid,
                          contributed);
        if (eg_eid >= 0) {
          if (eg_loc >= 0) {
            float4* g = &sm.dgrad[eg_loc];
            atomicAdd(&g->x, eg.x);
            atomicAdd(&g->y, eg.y);
            atomicAdd(&g->z, eg.z);
            atomicAdd(&g->w, eg.w);
          } else {
            float* g = A.v_edges + (long long)eg_eid * 4;
            atomicAdd(g, eg.x);
            atomicAdd(g + 1, eg.y);
            atomicAdd(g + 2, eg.z);
            atomicAdd(g + 3, eg.w);
          }
        }
      }
      if (!__any_sync(0xffffffffu, contributed)) continue;
#pragma unroll
      for (int c = 0; c < kAcc; ++c) {
        if (c == 5 && !STROKE) continue;
        if (c >= 6 && !collect) continue;
        const float v = warp_sum(acc[c]);
        if (lane == 0 && v != 0.0f) atomicAdd(&sm.pacc[pc][c], v);
      }
    }
    __syncthreads();
    // flush per-piece and per-edge accumulators
    for (int idx = tid; idx < np * kAcc; idx += kRT) {
      const int pc = idx / kAcc, c = idx - pc * kAcc;
      const float v = sm.pacc[pc][c];
      if (v == 0.0f) continue;
      const int pid = sm.piece[pc].pid;
      if (c < 3) atomicAdd(A.v_colors + pid * 3 + c, v);
      else if (c == 3) atomicAdd(A.v_opac + pid, v);
      else if (c == 4) atomicAdd(A.v_inv + pid, v);
      else if (c == 5) atomicAdd(A.v_sw + pid, v);
      else if (c < 9) { if (A.contrib) atomicAdd(A.contrib + pid * 3 + (c - 6), v); }
      else if (A.icontrib) atomicAdd(A.icontrib + sm.piece[pc].k, v);
    }
    const int ndl = sm.ndl;
    for (int d = tid; d < ndl; d += kRT) {
      const float4 g = sm.dgrad[d];
      if (g.x == 0.0f && g.y == 0.0f && g.z == 0.0f && g.w == 0.0f) continue;
      float* dst = A.v_edges + (long long)__float_as_int(sm.dB[d].w) * 4;
      atomicAdd(dst, g.x);
      atomicAdd(dst + 1, g.y);
      atomicAdd(dst + 2, g.z);
      atomicAdd(dst + 3, g.w);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host launch helpers

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
  dim3 grid(tbx, r1 - r0);
  if (!stroke && !bwd) raster_forward_kernel<false><<<grid, kRT, 0, st>>>(args);
  if (stroke && !bwd) raster_forward_kernel<true><<<grid, kRT, 0, st>>>(args);
  if (!stroke && bwd) raster_backward_kernel<false><<<grid, kRT, 0, st>>>(args);
  if (stroke && bwd) raster_backward_kernel<true><<<grid, kRT, 0, st>>>(args);
  return launch_status();
}

}  // namespace cs

using namespace cs;

extern "C" {

int cs_fill_forward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                    const float* edges_px, const int32_t* isect_edge_ranges,
                    const int32_t* prim_edge_offsets, const float* colors,
                    const float* opacities, const float* inv_sigma2s, const int32_t* fill_rules,
                    const float* background, float* out_img, float* final_Ts, int32_t* final_idx,
                    float* out_chw_clamped, int32_t img_height, int32_t img_width,
                    int32_t tile_row_begin, int32_t tile_row_end, void* stream) {
  if (img_height <= 0 || img_width <= 0 || !tile_bins || !out_img || !final_Ts || !final_idx ||
      (!isect_edge_ranges && !prim_edge_offsets))
    return CS_ERR_ARG;
  RasterArgs a{};
  a.pids = prim_ids_sorted;
  a.bins = tile_bins;
  a.edges = reinterpret_cast<const float4*>(edges_px);
  a.ranges = reinterpret_cast<const int2*>(isect_edge_ranges);
  a.eoffs = prim_edge_offsets;
  a.colors = colors;
  a.opac = opacities;
  a.inv_s2 = inv_sigma2s;
  a.rules = fill_rules;
  a.bg = background;
  a.out = out_img;
  a.fts = final_Ts;
  a.fidx = final_idx;
  a.out_chw = out_chw_clamped;
  return launch_raster(false, false, a, img_height, img_width, tile_row_begin, tile_row_end,
                       (cudaStream_t)stream);
}

int cs_fill_backward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                     const float* edges_px, const int32_t* isect_edge_ranges,
                     const int32_t* prim_edge_offsets, const float* colors,
                     const float* opacities, const float* inv_sigma2s, const int32_t* fill_rules,
                     const float* background, const float* final_Ts, const int32_t* final_idx,
                     const float* v_output, const float* out_img, const float* target_chw,
                     const float* mse_scale, float* v_edges, float* v_colors, float* v_opacities,
                     float* v_inv_sigma2s, float* curve_contrib_rgb, float* curve_isect_contrib,
                     int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                     int32_t tile_row_end, void* stream) {
  if (img_height <= 0 || img_width <= 0 || !tile_bins ||
      (!isect_edge_ranges && !prim_edge_offsets))
    return CS_ERR_ARG;
  if (!v_output && (!out_img || !target_chw || !mse_scale)) return CS_ERR_ARG;
  RasterArgs a{};
  a.pids = prim_ids_sorted;
  a.bins = tile_bins;
  a.edges = reinterpret_cast<const float4*>(edges_px);
  a.ranges = reinterpret_cast<const int2*>(isect_edge_ranges);
  a.eoffs = prim_edge_offsets;
  a.colors = colors;
  a.opac = opacities;
  a.inv_s2 = inv_sigma2s;
  a.rules = fill_rules;
  a.bg = background;
  a.fts_in = final_Ts;
  a.fidx_in = final_idx;
  a.v_out = v_output;
  a.out_img = out_img;
  a.tgt = target_chw;
  a.mse_scale = mse_scale;
  a.v_edges = v_edges;
  a.v_colors = v_colors;
  a.v_opac = v_opacities;
  a.v_inv = v_inv_sigma2s;
  a.contrib = curve_contrib_rgb;
  a.icontrib = curve_isect_contrib;
  return launch_raster(false, true, a, img_height, img_width, tile_row_begin, tile_row_end,
                       (cudaStream_t)stream);
}

int cs_stroke_forward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                      const float* edges_px, const int32_t* isect_edge_ranges,
                      const int32_t* prim_edge_offsets, const float* colors,
                      const float* opacities, const float* stroke_widths,
                      const float* inv_sigma2s, const float* background, float* out_img,
                      float* final_Ts, int32_t* final_idx, float* out_chw_clamped,
                      int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                      int32_t tile_row_end, void* stream) {
  if (img_height <= 0 || img_width <= 0 || !tile_bins || !out_img || !final_Ts || !final_idx ||
      (!isect_edge_ranges && !prim_edge_offsets))
    return CS_ERR_ARG;
  RasterArgs a{};
  a.pids = prim_ids_sorted;
  a.bins = tile_bins;
  a.edges = reinterpret_cast<const float4*>(edges_px);
  a.ranges = reinterpret_cast<const int2*>(isect_edge_ranges);
  a.eoffs = prim_edge_offsets;
  a.colors = colors;
  a.opac = opacities;
  a.inv_s2 = inv_sigma2s;
  a.sw = stroke_widths;
  a.bg = background;
  a.out = out_img;
  a.fts = final_Ts;
  a.fidx = final_idx;
  a.out_chw = out_chw_clamped;
  return launch_raster(true, false, a, img_height, img_width, tile_row_begin, tile_row_end,
                       (cudaStream_t)stream);
}

int cs_stroke_backward(const int32_t* prim_ids_sorted, const int32_t* tile_bins,
                       const float* edges_px, const int32_t* isect_edge_ranges,
                       const int32_t* prim_edge_offsets, const float* colors,
                       const float* opacities, const float* stroke_widths,
                       const float* inv_sigma2s, const float* background, const float* final_Ts,
                       const int32_t* final_idx, const float* v_output, const float* out_img,
                       const float* target_chw, const float* mse_scale, float* v_edges,
                       float* v_colors, float* v_opacities, float* v_stroke_widths,
                       float* v_inv_sigma2s, float* curve_contrib_rgb,
                       float* curve_isect_contrib, int32_t img_height, int32_t img_width,
                       int32_t tile_row_begin, int32_t tile_row_end, void* stream) {
  if (img_height <= 0 || img_width <= 0 || !tile_bins ||
      (!isect_edge_ranges && !prim_edge_offsets))
    return CS_ERR_ARG;
  if (!v_output && (!out_img || !target_chw || !mse_scale)) return CS_ERR_ARG;
  RasterArgs a{};
  a.pids = prim_ids_sorted;
  a.bins = tile_bins;
  a.edges = reinterpret_cast<const float4*>(edges_px);
  a.ranges = reinterpret_cast<const int2*>(isect_edge_ranges);
  a.eoffs = prim_edge_offsets;
  a.colors = colors;
  a.opac = opacities;
  a.inv_s2 = inv_sigma2s;
  a.sw = stroke_widths;
  a.bg = background;
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
  return launch_raster(true, true, a, img_height, img_width, tile_row_begin, tile_row_end,
                       (cudaStream_t)stream);
}

}  // extern "C"
