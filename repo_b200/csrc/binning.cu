// Projection, flattening and tile binning for the cubic renderer (sm_100a).
//
// Two families of entry points live here:
//  * stage kernels with the reference's signatures (project, flatten,
//    primitive ranges, intersect keys, tile bins, edge ranges) used by the
//    drop-in per-stage API;
//  * the fused B200 pipeline (cs_bin_count + cs_bin_sort): one warp per
//    primitive projects, bounds and flattens its segments and counts its
//    tiles; one CTA scans the per-tile counts into tile ranges; one warp per
//    primitive scatters its (depth, id) pairs into its tiles' ranges; one CTA
//    per tile sorts its pairs.  This replaces the reference's global 64-bit
//    key sort with per-tile sorts of (depth key, primitive id), which yields
//    exactly the order of a stable sort of the reference's keys.
#include "stage.cuh"

namespace cs {

// ---------------------------------------------------------------------------
// projection + exact cubic AABB + padded tile rectangle
// (manbo/ops/cubic_splatting.py:588-745).  Arithmetic is the reference's, in
// its written order; the pixel projection is one fused multiply-add, which is
// what the reference's compiled kernel does (pinned by golden vectors).

__device__ __forceinline__ void axis_extrema(float a, float b, float c, float d, float& mn,
                                             float& mx) {
  const float eps = kEps;
  float q2 = 3.0f * a;
  float q1 = 2.0f * b;
  float q0 = c;
  if ((q2 > eps) | (q2 < -eps)) {
    float disc = q1 * q1 - 4.0f * q2 * q0;
    if (disc >= -eps) {
      float sq = sqrtf(fmaxf(disc, 0.0f));
      float inv2q2 = 1.0f / (2.0f * q2);
      float t0 = (-q1 - sq) * inv2q2;
      float t1 = (-q1 + sq) * inv2q2;
      if ((t0 > 0.0f) & (t0 < 1.0f)) {
        float v = ((a * t0 + b) * t0 + c) * t0 + d;
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
      if ((t1 > 0.0f) & (t1 < 1.0f)) {
        float v = ((a * t1 + b) * t1 + c) * t1 + d;
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
    }
  } else if ((q1 > eps) | (q1 < -eps)) {
    float t = -q0 / q1;
    if ((t > 0.0f) & (t < 1.0f)) {
      float v = ((a * t + b) * t + c) * t + d;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
  }
}

__device__ __forceinline__ void project_points(const float* __restrict__ cn, float half_w,
                                               float half_h, float p[8]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    p[2 * k] = __fmaf_rn(cn[2 * k], half_w, half_w);
    p[2 * k + 1] = __fmaf_rn(cn[2 * k + 1], half_h, half_h);
  }
}

__device__ __forceinline__ void segment_rect(const float p[8], float stroke_w, float support_r,
                                             float aabb_pad, int aniso, int tbx, int tby,
                                             int rect[4]) {
  float p0x = p[0], p0y = p[1], p1x = p[2], p1y = p[3], p2x = p[4], p2y = p[5], p3x = p[6],
        p3y = p[7];
  float ax = -p0x + 3.0f * p1x - 3.0f * p2x + p3x;
  float bx = 3.0f * p0x - 6.0f * p1x + 3.0f * p2x;
  float cx = -3.0f * p0x + 3.0f * p1x;
  float ay = -p0y + 3.0f * p1y - 3.0f * p2y + p3y;
  float by = 3.0f * p0y - 6.0f * p1y + 3.0f * p2y;
  float cy = -3.0f * p0y + 3.0f * p1y;
  float min_x = fminf(p0x, p3x), max_x = fmaxf(p0x, p3x);
  float min_y = fminf(p0y, p3y), max_y = fmaxf(p0y, p3y);
  axis_extrema(ax, bx, cx, p0x, min_x, max_x);
  axis_extrema(ay, by, cy, p0y, min_y, max_y);
  float half_sw = fmaxf(0.0f, stroke_w) * 0.5f;
  float support = fmaxf(0.0f, support_r);
  if (aniso) {
    float chx = p3x - p0x, chy = p3y - p0y;
    float chord2 = chx * chx + chy * chy;
    float inv_chord = 1.0f / sqrtf(fmaxf(chord2, kEps));
    float nx = fmaxf(0.20f, fabsf(chy) * inv_chord);
    float ny = fmaxf(0.20f, fabsf(chx) * inv_chord);
    float radial = half_sw + support;
    float pad_x = aabb_pad + radial * nx;
    float pad_y = aabb_pad + radial * ny;
    min_x = min_x - pad_x;
    max_x = max_x + pad_x;
    min_y = min_y - pad_y;
    max_y = max_y + pad_y;
  } else {
    float pad_i = fmaxf(aabb_pad, support);
    min_x = min_x - half_sw - pad_i;
    min_y = min_y - half_sw - pad_i;
    max_x = max_x + half_sw + pad_i;
    max_y = max_y + half_sw + pad_i;
  }
  rect[0] = min(max(f2i_trunc_sat(min_x / 16.0f), 0), tbx);
  rect[1] = min(max(f2i_trunc_sat(min_y / 16.0f), 0), tby);
  rect[2] = min(max(f2i_trunc_sat(max_x / 16.0f + 1.0f), 0), tbx);
  rect[3] = min(max(f2i_trunc_sat(max_y / 16.0f + 1.0f), 0), tby);
}

// Bernstein point s of a pixel-space cubic: ((c0 b0 + c1 b1) + c2 b2) + c3 b3
// per coordinate (the summation order of torch's sum over the 4 control
// points, manbo/ops/cubic_splatting.py:1717).
__device__ __forceinline__ void bernstein_point(const float p[8], const float* __restrict__ basis,
                                                int S, int s, float& x, float& y) {
  float b0 = __ldg(basis + s), b1 = __ldg(basis + S + s), b2 = __ldg(basis + 2 * S + s),
        b3 = __ldg(basis + 3 * S + s);
  x = p[0] * b0 + p[2] * b1;
  x = x + p[4] * b2;
  x = x + p[6] * b3;
  y = p[1] * b0 + p[3] * b1;
  y = y + p[5] * b2;
  y = y + p[7] * b3;
}

__device__ __forceinline__ void store_point(float* __restrict__ edges, long long seg, int S, int s,
                                            float x, float y) {
  const long long E = S - 1;
  if (s > 0) *reinterpret_cast<float2*>(edges + (seg * E + s - 1) * 4 + 2) = make_float2(x, y);
  if (s < S - 1) *reinterpret_cast<float2*>(edges + (seg * E + s) * 4) = make_float2(x, y);
}

// ---------------------------------------------------------------------------
// stage kernels with reference signatures

__global__ void project_kernel(const float* __restrict__ cn, const float* __restrict__ sw,
                               const float* __restrict__ sr, float* __restrict__ cpx,
                               int* __restrict__ ranges, int* __restrict__ hits, long long n,
                               float half_w, float half_h, float pad, int aniso, int tbx, int tby) {
  long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n) return;
  float c[8], p[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] = cn[g * 8 + i];
  project_points(c, half_w, half_h, p);
#pragma unroll
  for (int i = 0; i < 8; ++i) cpx[g * 8 + i] = p[i];
  if (!ranges) return;  // projection only
  int r[4];
  segment_rect(p, sw ? sw[g] : 0.0f, sr ? sr[g] : 0.0f, pad, aniso, tbx, tby, r);
#pragma unroll
  for (int i = 0; i < 4; ++i) ranges[g * 4 + i] = r[i];
  if (hits) hits[g] = max(0, (r[2] - r[0]) * (r[3] - r[1]));
}

__global__ void flatten_kernel(const float* __restrict__ cpx, const float* __restrict__ basis,
                               float* __restrict__ edges, long long nseg, int S) {
  long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nseg * S) return;
  long long seg = q / S;
  int s = (int)(q - seg * S);
  float p[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = cpx[seg * 8 + i];
  float x, y;
  bernstein_point(p, basis, S, s, x, y);
  store_point(edges, seg, S, s, x, y);
}

__global__ void prim_ranges_kernel(const int* __restrict__ seg_ranges, const int* __restrict__ offs,
                                   int* __restrict__ pr, int* __restrict__ hits, long long np,
                                   int tbx, int tby) {
  long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= np) return;
  int s0 = offs[p], s1 = offs[p + 1];
  int r0 = 0, r1 = 0, r2 = 0, r3 = 0, h = 0;
  if (s1 > s0) {
    r0 = tbx; r1 = tby;
    for (int s = s0; s < s1; ++s) {
      r0 = min(r0, seg_ranges[s * 4 + 0]);
      r1 = min(r1, seg_ranges[s * 4 + 1]);
      r2 = max(r2, seg_ranges[s * 4 + 2]);
      r3 = max(r3, seg_ranges[s * 4 + 3]);
    }
    h = max(0, r2 - r0) * max(0, r3 - r1);
  }
  pr[p * 4 + 0] = r0; pr[p * 4 + 1] = r1; pr[p * 4 + 2] = r2; pr[p * 4 + 3] = r3;
  hits[p] = h;
}

__global__ void map_kernel(const int* __restrict__ ranges, const float* __restrict__ depths,
                           const int* __restrict__ cum, long long* __restrict__ ids,
                           int* __restrict__ pids, long long np, int tbx) {
  long long p = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (p >= np) return;
  int x0 = ranges[p * 4], y0 = ranges[p * 4 + 1], x1 = ranges[p * 4 + 2], y1 = ranges[p * 4 + 3];
  int w = x1 - x0, h = y1 - y0;
  if (w * h <= 0) return;
  long long base = p == 0 ? 0 : cum[p - 1];
  unsigned long long dk = depth_sort_key(depths[p]);
  for (int q = lane; q < w * h; q += 32) {
    int r = q / w, c = q - r * w;
    long long tile = (long long)(y0 + r) * tbx + x0 + c;
    ids[base + q] = (long long)(((unsigned long long)tile << 32) | dk);
    pids[base + q] = (int)p;
  }
}

__global__ void tile_bins_kernel(const long long* __restrict__ ids, long long n,
                                 int* __restrict__ bins) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int cur = (int)(ids[i] >> 32);
  if (i == 0) bins[cur * 2] = 0;
  if (i == n - 1) bins[cur * 2 + 1] = (int)n;
  if (i > 0) {
    int prev = (int)(ids[i - 1] >> 32);
    if (prev != cur) {
      bins[prev * 2 + 1] = (int)i;
      bins[cur * 2] = (int)i;
    }
  }
}

__global__ void edge_ranges_kernel(const int* __restrict__ pids, const int* __restrict__ eoffs,
                                   int* __restrict__ out, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int p = pids[i];
  out[i * 2] = eoffs[p];
  out[i * 2 + 1] = eoffs[p + 1];
}

// ---------------------------------------------------------------------------
// fused pipeline

// Zeroed before its first use; every cs_bin_count leaves the counts and the
// ticket zeroed again (the scan clears what it read).
struct BinWorkspace {
  int* tile_counts;     // [T] intersects per tile
  int* tile_ecounts;    // [T] edge slots per tile (each strip's record capacity)
  int* cursor;          // [T] scatter cursors
  unsigned* ticket;     // bin_prep CTAs done (the last one runs the scan)
};

__host__ __device__ inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

inline BinWorkspace bin_ws(void* base, long long ntiles) {
  BinWorkspace w;
  char* b = static_cast<char*>(base);
  const size_t a = align256(sizeof(int) * ntiles);
  w.tile_counts = reinterpret_cast<int*>(b);
  w.tile_ecounts = reinterpret_cast<int*>(b + a);
  w.cursor = reinterpret_cast<int*>(b + 2 * a);
  w.ticket = reinterpret_cast<unsigned*>(b + 3 * a);
  return w;
}

inline size_t bin_ws_size(long long ntiles) { return align256(sizeof(int) * ntiles) * 3 + 256; }

// Exclusive scans over the tiles [t0, t1) (the band) of the per-tile
// intersect counts into tile ranges [start, end) and of the per-tile edge-slot
// counts into staged-record ranges -- tile t owns kStrips consecutive lists of
// capacity ecount[t] each, so tile_dlist[t] = (first record, ecount[t]) and
// the record bound is kStrips * sum(ecount) -- by one CTA of any multiple of
// 32 threads.  Tiles outside the band read as empty.  If a total exceeds its
// capacity every range is written empty and the status is set.  The counts
// are zeroed as they are consumed.  counts (with bins, cursor) or ecounts
// (with dlr) may be NULL.
__device__ void scan_tiles(int* __restrict__ counts, int* __restrict__ ecounts,
                           int* __restrict__ bins, int* __restrict__ dlr,
                           int* __restrict__ cursor, int* __restrict__ counters, long long t0,
                           long long t1, long long nt, long long icap, long long dcap) {
  __shared__ int wa[32], wb[32];
  __shared__ long long s_ta, s_tb;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nthr = blockDim.x, nw = nthr >> 5;
  const long long n = t1 - t0;
  const long long chunk = (n + nthr - 1) / nthr;
  const long long b = t0 + tid * chunk, e = min(t1, b + chunk);
  // up to kScanCache counts per thread are loaded at once and kept in
  // registers for the second walk (one memory round trip instead of two
  // per count)
  constexpr int kScanCache = 8;
  const bool cached = chunk <= kScanCache;
  int ca[kScanCache], cb[kScanCache];
  int la = 0, lb = 0;
  if (cached) {
#pragma unroll
    for (int j = 0; j < kScanCache; ++j) {
      const long long i = b + j;
      ca[j] = (counts && i < e) ? __ldcg(counts + i) : 0;
      cb[j] = (ecounts && i < e) ? __ldcg(ecounts + i) : 0;
    }
#pragma unroll
    for (int j = 0; j < kScanCache; ++j) {
      la += ca[j];
      lb += cb[j];
    }
  } else {
    for (long long i = b; i < e; ++i) {
      if (counts) la += __ldcg(counts + i);
      if (ecounts) lb += __ldcg(ecounts + i);
    }
  }
  int ia = warp_incl_scan(la, lane), ib = warp_incl_scan(lb, lane);
  if (lane == 31) {
    wa[wid] = ia;
    wb[wid] = ib;
  }
  __syncthreads();
  if (wid == 0) {
    const int va = lane < nw ? wa[lane] : 0, vb = lane < nw ? wb[lane] : 0;
    const int xa = warp_incl_scan(va, lane), xb = warp_incl_scan(vb, lane);
    wa[lane] = xa - va;
    wb[lane] = xb - vb;
    if (lane == 31) {
      s_ta = xa;
      s_tb = (long long)kStrips * xb;
      if (counts) counters[0] = xa;
      if (ecounts) counters[2] = (int)min((long long)kStrips * xb, (long long)INT32_MAX);
      if ((counts && xa > icap) || (ecounts && s_tb > dcap)) counters[1] = CS_ERR_CAPACITY;
    }
  }
  __syncthreads();
  const bool overflow = (counts && s_ta > icap) || (ecounts && s_tb > dcap);
  int ra = wa[wid] + ia - la, rb = wb[wid] + ib - lb;
  if (cached) {
#pragma unroll
    for (int j = 0; j < kScanCache; ++j) {
      const long long i = b + j;
      if (i >= e) break;
      if (counts) {
        const int c = overflow ? 0 : ca[j];
        counts[i] = 0;
        cursor[i] = ra;
        bins[2 * i] = c > 0 ? ra : 0;
        bins[2 * i + 1] = c > 0 ? ra + c : 0;
        ra += c;
      }
      if (ecounts) {
        const int c = overflow ? 0 : cb[j];
        ecounts[i] = 0;
        dlr[2 * i] = c > 0 ? kStrips * rb : 0;
        dlr[2 * i + 1] = c > 0 ? c : 0;
        rb += c;
      }
    }
  }
  for (long long i = cached ? e : b; i < e; ++i) {
    if (counts) {
      const int c = overflow ? 0 : __ldcg(counts + i);
      counts[i] = 0;
      cursor[i] = ra;
      bins[2 * i] = c > 0 ? ra : 0;
      bins[2 * i + 1] = c > 0 ? ra + c : 0;
      ra += c;
    }
    if (ecounts) {
      const int c = overflow ? 0 : __ldcg(ecounts + i);
      ecounts[i] = 0;
      dlr[2 * i] = c > 0 ? kStrips * rb : 0;
      dlr[2 * i + 1] = c > 0 ? c : 0;
      rb += c;
    }
  }
  for (long long i = tid; i < nt; i += nthr) {  // a band: the other tiles are empty
    if (i >= t0 && i < t1) continue;
    if (counts) bins[2 * i] = bins[2 * i + 1] = 0;
    if (ecounts) dlr[2 * i] = dlr[2 * i + 1] = 0;
  }
}

// The scan on its own (the per-stage staging path): one CTA of 1024.
__global__ void __launch_bounds__(1024) bin_scan_kernel(int* __restrict__ counts,
                                                        int* __restrict__ ecounts,
                                                        int* __restrict__ bins,
                                                        int* __restrict__ dlr,
                                                        int* __restrict__ cursor,
                                                        int* __restrict__ counters, long long t0,
                                                        long long t1, long long icap,
                                                        long long dcap) {
  scan_tiles(counts, ecounts, bins, dlr, cursor, counters, t0, t1, t1, icap, dcap);
}

// Normalised control points of segment `seg`: from cubics_norm [n, 4, 2], or,
// when ring != NULL, from the ring parameterisation of closed paths (segment k
// of a path = ring points 3k .. 3k+3 mod 3G, normalised as ring / (W/2, H/2) - 1,
// the same arithmetic as cs_ring_to_cubics).
__device__ __forceinline__ void load_segment(const float* __restrict__ cn,
                                             const float* __restrict__ ring, int G, float half_w,
                                             float half_h, long long seg, float c[8]) {
  if (!ring) {
#pragma unroll
    for (int k = 0; k < 8; ++k) c[k] = cn[seg * 8 + k];
    return;
  }
  const long long path = seg / G;
  const int k = (int)(seg - path * G);
  const float2* rp = reinterpret_cast<const float2*>(ring) + path * 3 * G;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int r = 3 * k + j;
    if (r >= 3 * G) r -= 3 * G;
    const float2 v = rp[r];
    c[2 * j] = v.x / half_w - 1.0f;
    c[2 * j + 1] = v.y / half_h - 1.0f;
  }
}

// One warp: project + bound every segment of primitive p, union the rects,
// flatten the segments (unless pre-flattened), and count the primitive in
// its tiles within the band.
__device__ __forceinline__ void prep_primitive(
    const float* __restrict__ cn, const float* __restrict__ ring, int ring_g,
    const int* __restrict__ offs, const int* __restrict__ peo, int* __restrict__ peo_out,
    const float* __restrict__ aa, const float* __restrict__ sw, const float* __restrict__ basis,
    float* __restrict__ cpx, float* __restrict__ edges, int* __restrict__ pr,
    int* __restrict__ hits, int* __restrict__ tile_counts, int* __restrict__ tile_ecounts,
    int* __restrict__ status, long long p, long long np, long long nseg_total, int S,
    float half_w, float half_h, int tbx, int tby, int r0, int r1, float pad, int aniso) {
  int lane = threadIdx.x & 31;
  int s0 = offs[p], s1 = offs[p + 1];
  if (peo_out && lane == 0) {  // primitive edge offsets of the uniform flatten: offs * (S - 1)
    peo_out[p] = (int)((long long)s0 * (S - 1));
    if (p == np - 1) peo_out[np] = (int)((long long)s1 * (S - 1));
  }
  // CSR offsets must start at 0, end at the segment count and not decrease;
  // a bad primitive is reported and treated as empty (no out-of-bounds reads).
  const bool bad = s0 < 0 || s1 < s0 || s1 > nseg_total || (p == 0 && s0 != 0) ||
                   (p == np - 1 && s1 != nseg_total);
  if (bad) {
    if (lane == 0 && status) atomicExch(status, CS_ERR_ARG);
    s1 = s0 = max(0, min(s0, (int)nseg_total));
  }
  float w = fmaxf(aa[p], 1e-4f);
  float support = w * 3.0f;
  float stroke = sw ? sw[p] : 0.0f;
  int mnx = tbx, mny = tby, mxx = 0, mxy = 0;
  for (int i = s0 + lane; i < s1; i += 32) {
    float c[8], q[8];
    load_segment(cn, ring, ring_g, half_w, half_h, i, c);
    project_points(c, half_w, half_h, q);
    float4* dst = reinterpret_cast<float4*>(cpx + (long long)i * 8);
    dst[0] = make_float4(q[0], q[1], q[2], q[3]);
    dst[1] = make_float4(q[4], q[5], q[6], q[7]);
    int r[4];
    segment_rect(q, stroke, support, pad, aniso, tbx, tby, r);
    mnx = min(mnx, r[0]); mny = min(mny, r[1]); mxx = max(mxx, r[2]); mxy = max(mxy, r[3]);
  }
  mnx = warp_min_i(mnx); mny = warp_min_i(mny); mxx = warp_max_i(mxx); mxy = warp_max_i(mxy);
  int nseg = s1 - s0;
  if (nseg <= 0) { mnx = mny = mxx = mxy = 0; }
  int count = nseg > 0 ? max(0, mxx - mnx) * max(0, mxy - mny) : 0;
  if (lane == 0) {
    *reinterpret_cast<int4*>(pr + p * 4) = make_int4(mnx, mny, mxx, mxy);
    hits[p] = count;
  }
  // edges are needed only by the band's tiles: a primitive whose tile rows
  // miss the band is not flattened
  const bool in_band = max(mny, r0) < min(mxy, r1) && mnx < mxx;
  const int npts = (in_band && !peo) ? nseg * S : 0;
  for (int q = lane; q < npts; q += 32) {
    int si = q / S;
    int s = q - si * S;
    long long seg = s0 + si;
    float c[8], pp[8];
    load_segment(cn, ring, ring_g, half_w, half_h, seg, c);
    project_points(c, half_w, half_h, pp);
    float x, y;
    bernstein_point(pp, basis, S, s, x, y);
    store_point(edges, seg, S, s, x, y);
  }
  int nedge = nseg * (S - 1);
  if (peo) {  // pre-flattened: the primitive's edges are peo[p] .. peo[p + 1]
    nedge = peo[p + 1] - peo[p];
    if (nedge < 0 || peo[p] < 0) {
      if (lane == 0 && status) atomicExch(status, CS_ERR_ARG);
      nedge = 0;
    }
  }
  int y0 = max(mny, r0), y1 = min(mxy, r1);
  int wdt = mxx - mnx, hgt = y1 - y0;
  if (wdt > 0 && hgt > 0) {
    for (int q = lane; q < wdt * hgt; q += 32) {
      int rr = q / wdt, cc = q - rr * wdt;
      const long long t = (long long)(y0 + rr) * tbx + mnx + cc;
      atomicAdd(tile_counts + t, 1);
      atomicAdd(tile_ecounts + t, nedge);
    }
  }
}

// One warp per primitive: project + bound every segment, union the rects,
// flatten all segments into edges (unless peo gives pre-flattened edges with
// their CSR offsets), and add the primitive to the intersect and edge-slot
// counts of its tiles within the band of tile rows [r0, r1).
constexpr int kPrepThreads = 512;  // one warp per primitive; the last CTA to finish scans the tiles

__global__ void __launch_bounds__(kPrepThreads) bin_prep_kernel(
    const float* __restrict__ cn, const float* __restrict__ ring, int ring_g,
    const int* __restrict__ offs, const int* __restrict__ peo, int* __restrict__ peo_out,
    const float* __restrict__ aa,
    const float* __restrict__ sw, const float* __restrict__ basis, float* __restrict__ cpx,
    float* __restrict__ edges, int* __restrict__ pr, int* __restrict__ hits,
    BinWorkspace ws, int* __restrict__ bins, int* __restrict__ dlr, int* __restrict__ counters,
    long long np, long long nseg_total, int S, float half_w, float half_h, int tbx, int tby,
    int r0, int r1, float pad, int aniso, long long icap, long long dcap) {
  const long long p = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (p < np) prep_primitive(cn, ring, ring_g, offs, peo, peo_out, aa, sw, basis, cpx, edges, pr,
                             hits, ws.tile_counts, ws.tile_ecounts, counters + 1, p, np,
                             nseg_total, S, half_w, half_h, tbx, tby, r0, r1, pad, aniso);
  // the last CTA to finish scans the counts
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ws.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const long long nt = (long long)tbx * tby;
  const long long t0 = (long long)r0 * tbx, t1 = (long long)max(r0, r1) * tbx;
  scan_tiles(ws.tile_counts, ws.tile_ecounts, bins, dlr, ws.cursor, counters, t0, t1, nt, icap,
             dcap);
  if (threadIdx.x == 0) *ws.ticket = 0u;
}

// One warp per primitive: scatter (depth key << 32 | primitive id) into the
// primitive's tiles' ranges (unordered within a tile).
__global__ void __launch_bounds__(256) bin_scatter_kernel(
    const int* __restrict__ pr, const float* __restrict__ depths, int* __restrict__ cursor,
    unsigned long long* __restrict__ pairs, const int* __restrict__ counters, long long np,
    int tbx, long long capacity, int r0, int r1, int* __restrict__ lists) {
  long long p = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  // the staging pass appends to the dispatch lists: start them empty
  if (lists && blockIdx.x == 0 && threadIdx.x < kUnitBuckets) lists[threadIdx.x] = 0;
  if (p >= np) return;
  if (counters[0] > capacity) return;  // overflow reported by the scan
  int4 r = *reinterpret_cast<const int4*>(pr + p * 4);
  int y0 = max(r.y, r0), y1 = min(r.w, r1);
  int wdt = r.z - r.x, hgt = y1 - y0;
  if (wdt <= 0 || hgt <= 0) return;
  unsigned long long v = ((unsigned long long)depth_sort_key(depths[p]) << 32) | (unsigned)p;
  for (int q = lane; q < wdt * hgt; q += 32) {
    int rr = q / wdt, cc = q - rr * wdt;
    int slot = atomicAdd(cursor + (long long)(y0 + rr) * tbx + r.x + cc, 1);
    if (slot < capacity) pairs[slot] = v;
  }
}

constexpr int kSortThreads = 256;   // one CTA per tile for the sort and the staging
constexpr int kSortSmem = 4096;     // pairs sorted in shared memory (more: rank sort)
constexpr int kStageU = 2;          // edge slots per thread per staging round

__device__ __forceinline__ void emit_sorted(unsigned long long v, long long tile, long long pos,
                                            int* __restrict__ pids, long long* __restrict__ ids) {
  pids[pos] = (int)(v & 0xffffffffull);
  if (ids) ids[pos] = (long long)(((unsigned long long)tile << 32) | (v >> 32));
}

// Sort one tile's pairs ascending (CTA of kSortThreads); pairs are unique.
__device__ void sort_tile(unsigned long long* __restrict__ pairs, int start, int n, long long tile,
                          const float* __restrict__ depths, int* __restrict__ pids,
                          long long* __restrict__ ids, unsigned long long* s) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (n <= 32) {
    if (tid < 32) {
      unsigned long long v = lane < n ? pairs[start + lane] : ~0ull;
#pragma unroll
      for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
          unsigned long long o = __shfl_xor_sync(0xffffffffu, v, j);
          bool up = (lane & k) == 0;
          bool lower = (lane & j) == 0;
          v = (lower == up) ? min(v, o) : max(v, o);
        }
      }
      if (lane < n) emit_sorted(v, tile, start + lane, pids, ids);
    }
    return;
  }
  if (n <= kSortSmem) {
    int m = 64;
    while (m < n) m <<= 1;
    for (int i = tid; i < m; i += kSortThreads) s[i] = i < n ? pairs[start + i] : ~0ull;
    __syncthreads();
    for (int k = 2; k <= m; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < m; i += kSortThreads) {
          int ixj = i ^ j;
          if (ixj > i) {
            unsigned long long a = s[i], b = s[ixj];
            bool asc = (i & k) == 0;
            if ((a > b) == asc) { s[i] = b; s[ixj] = a; }
          }
        }
        __syncthreads();
      }
    }
    for (int i = tid; i < n; i += kSortThreads) emit_sorted(s[i], tile, start + i, pids, ids);
    return;
  }
  // Large tile: rank each pair by counting smaller pairs, then rebuild keys.
  for (int i = tid; i < n; i += kSortThreads) {
    unsigned long long v = pairs[start + i];
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += pairs[start + j] < v;
    pids[start + rank] = (int)(v & 0xffffffffull);
  }
  __syncthreads();
  if (ids) {
    for (int i = tid; i < n; i += kSortThreads) {
      int p = pids[start + i];
      ids[start + i] = (long long)(((unsigned long long)tile << 32) |
                                   (unsigned long long)depth_sort_key(depths[p]));
    }
  }
}

struct StageIO {
  const int* pids;
  const float4* edges;
  const int2* ranges;   // per intersect [eb, ee) or NULL
  const int* eoffs;     // per primitive edge offsets (when ranges is NULL)
  const float* colors;
  const float* opac;
  const float* inv_s2;
  const int* rules;
  const float* sw;      // stroke widths: non-NULL selects stroke mode
  int2* dlr;
  IMeta* imeta;
  int* rowoff;
  int2* istrip;         // per intersect and strip: (first record, record count)
  DEntry* dl;
  int tbx;
};

__device__ __forceinline__ void isect_edges(const StageIO& io, int k, int pid, int& eb, int& ee) {
  if (io.ranges) {
    const int2 r = io.ranges[k];
    eb = r.x;
    ee = r.y;
  } else {
    eb = io.eoffs[pid];
    ee = io.eoffs[pid + 1];
  }
}

// Shared state of stage_tile for one chunk of up to kSortThreads intersects.
struct StageShared {
  int sstart[kSortThreads + 1];  // first edge slot of each intersect; [m] = slot total
  int eb[kSortThreads];          // first edge of each intersect
  float dthr[kSortThreads];      // culling distance of each intersect
  int dstart[kStrips][kSortThreads + 1];  // first record per strip; [m] = chunk end
  unsigned bal[kStrips][kStageU][kSortThreads / 32];  // near ballots of the round
  int pre[kStrips][kStageU][kSortThreads / 32];       // their exclusive prefix counts
  int wsum[kSortThreads / 32];
  int total[kStrips];
};

// Classify the edges of intersects [rs, re) of one tile and write its staged
// records (CTA of kSortThreads; see stage.cuh), in one pass.  The intersects
// are taken in chunks of kSortThreads, one per thread for their attributes;
// the chunk's edges are laid out as consecutive slots (intersect-major, edge
// order within), which every thread walks kStageU slots per round.  A near
// edge's position in a strip's list is the number of slots before it that are
// near that strip (ballots and a prefix over the round's warps), which keeps
// (intersect, edge) order; an intersect's first record in a strip is that
// count at its first slot.  Strip st's list starts at dbase + st * stride.
// Far edges right of the tile add to the intersect's per-row winding
// accumulators in shared memory (`rows`, kSortThreads x 32 ints: 16 winding
// sums, 16 counts).  Returns the strips' record totals (in every thread).
template <bool STROKE>
__device__ void stage_tile(const StageIO& io, long long tile, int rs, int re, int dbase,
                           int stride, StageShared& sh, int (*rows)[32], int totals[kStrips]) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int nw = kSortThreads / 32;
  constexpr int kRound = kSortThreads * kStageU;
  const float bx0 = (float)((tile % io.tbx) * kTile) + 0.5f;
  const float by0 = (float)((tile / io.tbx) * kTile) + 0.5f;
  const unsigned lt = (1u << lane) - 1u;
  int near_base[kStrips];
#pragma unroll
  for (int st = 0; st < kStrips; ++st) near_base[st] = 0;
  for (int c0 = rs; c0 < re; c0 += kSortThreads) {
    const int m = min(kSortThreads, re - c0);
    // per intersect: attributes, edge range, slot count
    IMeta im;
    int ne = 0;
    if (tid < m) {
      const int k = c0 + tid;
      const int pid = io.pids[k];
      int eb, ee;
      isect_edges(io, k, pid, eb, ee);
      intersect_attrs<STROKE>(pid, io.colors, io.opac, io.inv_s2, io.rules, io.sw, im);
      ne = max(0, ee - eb);
      sh.eb[tid] = eb;
      sh.dthr[tid] = im.dthr;
      if (!STROKE) {
#pragma unroll
        for (int r = 0; r < 32; ++r) rows[tid][r] = 0;
      }
    }
    const int incl = warp_incl_scan(ne, lane);
    if (lane == 31) sh.wsum[wid] = incl;
    __syncthreads();
    int wbase = 0, total = 0;
#pragma unroll
    for (int w2 = 0; w2 < nw; ++w2) {
      const int v = sh.wsum[w2];
      wbase += w2 < wid ? v : 0;
      total += v;
    }
    if (tid < m) sh.sstart[tid] = wbase + incl - ne;
    if (tid == 0) sh.sstart[m] = total;
    __syncthreads();
    for (int rb = 0; rb < total; rb += kRound) {
      int kk[kStageU], ee_[kStageU];
      float4 E[kStageU];
#pragma unroll
      for (int u = 0; u < kStageU; ++u) {
        const int j = rb + u * kSortThreads + tid;
        kk[u] = -1;
        ee_[u] = 0;
        if (j < total) {
          int lo = 0, hi = m;  // last intersect whose first slot is <= j
          while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (sh.sstart[mid] <= j) lo = mid; else hi = mid;
          }
          kk[u] = lo;
          ee_[u] = sh.eb[lo] + (j - sh.sstart[lo]);
        }
      }
#pragma unroll
      for (int u = 0; u < kStageU; ++u)
        E[u] = kk[u] >= 0 ? __ldg(io.edges + ee_[u]) : make_float4(0.f, 0.f, 0.f, 0.f);
      unsigned nm[kStageU], bal[kStrips][kStageU];
#pragma unroll
      for (int u = 0; u < kStageU; ++u) {
        nm[u] = kk[u] >= 0 ? edge_near_strips(E[u], sh.dthr[kk[u]], bx0, by0) : 0u;
#pragma unroll
        for (int st = 0; st < kStrips; ++st) {
          bal[st][u] = __ballot_sync(0xffffffffu, (nm[u] >> st) & 1u);
          if (lane == 0) sh.bal[st][u][wid] = bal[st][u];
        }
        if (!STROKE && kk[u] >= 0) {
          unsigned rr = far_right_rows(E[u], bx0, by0) & ~strip_rows(nm[u]);
          if (rr) {
            const int dir = (E[u].w - E[u].y) > 0.0f ? 1 : -1;
            while (rr) {
              const int r = __ffs(rr) - 1;
              rr &= rr - 1u;
              atomicAdd(&rows[kk[u]][r], dir);
              atomicAdd(&rows[kk[u]][16 + r], 1);
            }
          }
        }
      }
      __syncthreads();
      if (wid < kStrips) {  // warp st: exclusive prefix of strip st's (u, warp) counts
        const int st = wid;
        const int v = lane < kStageU * nw ? __popc(sh.bal[st][lane / nw][lane % nw]) : 0;
        const int x = warp_incl_scan(v, lane);
        if (lane < kStageU * nw) sh.pre[st][lane / nw][lane % nw] = x - v;
        if (lane == 31) sh.total[st] = x;
      }
      __syncthreads();
#pragma unroll
      for (int u = 0; u < kStageU; ++u) {
        if (nm[u]) {
          const DEntry rec = make_entry(E[u], ee_[u]);
#pragma unroll
          for (int st = 0; st < kStrips; ++st) {
            if ((nm[u] >> st) & 1u) {
              const int pos = near_base[st] + sh.pre[st][u][wid] + __popc(bal[st][u] & lt);
              io.dl[dbase + st * stride + pos] = rec;
            }
          }
        }
      }
      if (tid < m) {
        const int sl = sh.sstart[tid] - rb;
        if (sl >= 0 && sl < kRound && sh.sstart[tid] < total) {
          const int u = sl / kSortThreads, w2 = (sl % kSortThreads) >> 5, l = sl & 31;
          const unsigned below = (1u << l) - 1u;
#pragma unroll
          for (int st = 0; st < kStrips; ++st)
            sh.dstart[st][tid] = near_base[st] + sh.pre[st][u][w2] + __popc(sh.bal[st][u][w2] & below);
        }
      }
#pragma unroll
      for (int st = 0; st < kStrips; ++st) near_base[st] += sh.total[st];
      __syncthreads();
    }
    // intersects with no slot left (empty, at the end of the chunk)
    if (tid < m && sh.sstart[tid] >= total) {
#pragma unroll
      for (int st = 0; st < kStrips; ++st) sh.dstart[st][tid] = near_base[st];
    }
    if (tid == 0) {
#pragma unroll
      for (int st = 0; st < kStrips; ++st) sh.dstart[st][m] = near_base[st];
    }
    __syncthreads();
    if (tid < m) {
      const int k = c0 + tid;
      int4* dst = reinterpret_cast<int4*>(io.imeta + k);
      dst[0] = make_int4(0, 0, im.pid, im.rule);
      dst[1] = make_int4(__float_as_int(im.c0), __float_as_int(im.c1), __float_as_int(im.c2),
                         __float_as_int(im.op));
      dst[2] = make_int4(__float_as_int(im.a), __float_as_int(im.b), __float_as_int(im.dthr), 0);
      int4* sr = reinterpret_cast<int4*>(io.istrip + (long long)k * kStrips);
      int v[2 * kStrips];
#pragma unroll
      for (int st = 0; st < kStrips; ++st) {
        v[2 * st] = sh.dstart[st][tid];
        v[2 * st + 1] = sh.dstart[st][tid + 1] - sh.dstart[st][tid];
      }
      sr[0] = make_int4(v[0], v[1], v[2], v[3]);
      sr[1] = make_int4(v[4], v[5], v[6], v[7]);
    }
    if (!STROKE) {
      for (int q = tid; q < m * 16; q += kSortThreads) {
        const int t = q >> 4, r = q & 15;
        io.rowoff[(long long)(c0 + t) * 16 + r] = pack_row(rows[t][r], rows[t][16 + r]);
      }
    }
    __syncthreads();  // shared state is reused by the next chunk
  }
#pragma unroll
  for (int st = 0; st < kStrips; ++st) totals[st] = near_base[st];
}

// Work estimate of a strip for dispatch ordering, in half-records: its staged
// records plus two and a half per intersect (an intersect's compositing costs
// about as much as two and a half records).
__device__ __forceinline__ int strip_weight(int records, int intersects) {
  return intersects > 0 ? 2 * records + 5 * intersects : 0;
}

// One CTA per tile: sort the tile's pairs and emit primitive ids and
// reference-format intersect ids; then, when staging outputs are given,
// classify the tile's edges into its strips' records and file each strip into
// the dispatch lists by its work estimate (one atomic per strip).
template <bool STROKE>
__global__ void __launch_bounds__(kSortThreads) bin_tile_kernel(
    const int* __restrict__ bins, const float* __restrict__ depths,
    unsigned long long* __restrict__ pairs, int* __restrict__ pids, long long* __restrict__ ids,
    const int* __restrict__ counters, long long icap, long long dcap, int r0, StageIO io,
    int* __restrict__ lists) {
  // the sort buffer is reused for the staging row accumulators
  static_assert(sizeof(unsigned long long) * kSortSmem >= sizeof(int) * kSortThreads * 32,
                "row accumulators must fit the sort buffer");
  __shared__ __align__(16) unsigned long long s[kSortSmem];
  __shared__ StageShared sh;
  const long long tile = (long long)(r0 + blockIdx.y) * io.tbx + blockIdx.x;
  const int unit0 = kStrips * (blockIdx.y * gridDim.x + blockIdx.x);
  const int start = bins[2 * tile], end = bins[2 * tile + 1];
  const int n = end - start;
  const bool sorted = n > 0 && counters[0] <= icap;  // on overflow the pairs were not all written
  if (sorted) sort_tile(pairs, start, n, tile, depths, pids, ids, s);
  if (!io.imeta) return;
  int totals[kStrips] = {0, 0, 0, 0};
  if (sorted && counters[2] <= dcap) {
    __syncthreads();
    const int2 dl = io.dlr[tile];
    stage_tile<STROKE>(io, tile, start, end, dl.x, dl.y, sh, reinterpret_cast<int (*)[32]>(s),
                       totals);
  }
  if (lists && threadIdx.x < kStrips) {
    int t = 0;
#pragma unroll
    for (int st = 0; st < kStrips; ++st) t = threadIdx.x == st ? totals[st] : t;
    append_unit(lists, kStrips * gridDim.x * gridDim.y, unit0 + threadIdx.x,
                sorted ? strip_weight(t, n) : 0);
  }
}

// Standalone staging for a reference-format intersect list: per-tile edge-slot
// bound (one warp per tile) ...
__global__ void tile_esum_kernel(const int* __restrict__ bins, const int* __restrict__ pids,
                                 const int2* __restrict__ ranges, const int* __restrict__ eoffs,
                                 int* __restrict__ ecounts, long long nt) {
  const long long t = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= nt) return;
  const int rs = bins[2 * t], re = bins[2 * t + 1];
  int acc = 0;
  for (int k = rs + lane; k < re; k += 32) {
    if (ranges) {
      const int2 r = ranges[k];
      acc += max(0, r.y - r.x);
    } else {
      const int p = pids[k];
      acc += max(0, eoffs[p + 1] - eoffs[p]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) ecounts[t] = acc;
}

// ... and the staging pass itself (one CTA per tile).
template <bool STROKE>
__global__ void __launch_bounds__(kSortThreads) tile_stage_kernel(const int* __restrict__ bins,
                                                                  const int* __restrict__ counters,
                                                                  long long dcap, StageIO io,
                                                                  int* __restrict__ lists) {
  __shared__ int s_row[STROKE ? 1 : kSortThreads][32];
  __shared__ StageShared sh;
  const long long tile = (long long)blockIdx.y * io.tbx + blockIdx.x;
  const int unit0 = kStrips * (blockIdx.y * gridDim.x + blockIdx.x);
  const int rs = bins[2 * tile], re = bins[2 * tile + 1];
  int totals[kStrips] = {0, 0, 0, 0};
  const bool staged = re > rs && counters[2] <= dcap;
  if (staged) {
    const int2 dl = io.dlr[tile];
    stage_tile<STROKE>(io, tile, rs, re, dl.x, dl.y, sh, s_row, totals);
  }
  if (lists && threadIdx.x < kStrips) {
    int t = 0;
#pragma unroll
    for (int st = 0; st < kStrips; ++st) t = threadIdx.x == st ? totals[st] : t;
    append_unit(lists, kStrips * gridDim.x * gridDim.y, unit0 + threadIdx.x,
                staged ? strip_weight(t, re - rs) : 0);
  }
}

}  // namespace cs

using namespace cs;

extern "C" {

const char* cs_version(void) { return "cubicsplat_b200 0.1.0 sm_100a"; }

int cs_project_cubics(const float* cubics_norm, const float* stroke_widths,
                      const float* support_radii, float* cubics_px, int32_t* tile_ranges,
                      int32_t* num_tiles_hit, int64_t num_curves, int32_t img_height,
                      int32_t img_width, int32_t block_x, int32_t block_y, float aabb_pad,
                      int32_t aniso, void* stream) {
  if (block_x != kTile || block_y != kTile) return CS_ERR_UNSUPPORTED;
  if (num_curves < 0 || img_height <= 0 || img_width <= 0) return CS_ERR_ARG;
  if (num_curves == 0) return CS_OK;
  if (!cubics_norm || !cubics_px) return CS_ERR_ARG;
  int tbx = (img_width + kTile - 1) / kTile, tby = (img_height + kTile - 1) / kTile;
  project_kernel<<<ceil_div(num_curves, 256), 256, 0, (cudaStream_t)stream>>>(
      cubics_norm, stroke_widths, support_radii, cubics_px, tile_ranges, num_tiles_hit,
      num_curves, 0.5f * (float)img_width, 0.5f * (float)img_height, aabb_pad, aniso, tbx, tby);
  return launch_status();
}

int cs_flatten_bernstein(const float* cubics_px, const float* basis, float* edges_px,
                         int64_t num_segments, int32_t samples, void* stream) {
  if (samples < 2 || num_segments < 0) return CS_ERR_ARG;
  if (num_segments == 0) return CS_OK;
  long long n = num_segments * samples;
  flatten_kernel<<<ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(cubics_px, basis, edges_px,
                                                                     num_segments, samples);
  return launch_status();
}

int cs_primitive_tile_ranges(const int32_t* seg_tile_ranges, const int32_t* prim_seg_offsets,
                             int32_t* prim_tile_ranges, int32_t* num_tiles_hit,
                             int64_t num_primitives, int32_t tile_bound_x, int32_t tile_bound_y,
                             void* stream) {
  if (num_primitives < 0) return CS_ERR_ARG;
  if (num_primitives == 0) return CS_OK;
  prim_ranges_kernel<<<ceil_div(num_primitives, 256), 256, 0, (cudaStream_t)stream>>>(
      seg_tile_ranges, prim_seg_offsets, prim_tile_ranges, num_tiles_hit, num_primitives,
      tile_bound_x, tile_bound_y);
  return launch_status();
}

int cs_map_cubic_to_intersects(const int32_t* tile_ranges, const float* depths,
                               const int32_t* cum_tiles_hit, int64_t* isect_ids,
                               int32_t* prim_ids, int64_t num_primitives, int32_t tile_bound_x,
                               void* stream) {
  if (num_primitives < 0) return CS_ERR_ARG;
  if (num_primitives == 0) return CS_OK;
  map_kernel<<<ceil_div(num_primitives * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      tile_ranges, depths, cum_tiles_hit, reinterpret_cast<long long*>(isect_ids), prim_ids,
      num_primitives, tile_bound_x);
  return launch_status();
}

int cs_tile_bin_edges(const int64_t* isect_ids_sorted, int64_t num_intersects,
                      int32_t* tile_bins, int64_t num_tiles, void* stream) {
  if (num_intersects < 0 || num_tiles <= 0) return CS_ERR_ARG;
  cudaMemsetAsync(tile_bins, 0, sizeof(int32_t) * 2 * num_tiles, (cudaStream_t)stream);
  if (num_intersects == 0) return launch_status();
  tile_bins_kernel<<<ceil_div(num_intersects, 256), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const long long*>(isect_ids_sorted), num_intersects, tile_bins);
  return launch_status();
}

int cs_isect_edge_ranges(const int32_t* prim_ids_sorted, const int32_t* prim_edge_offsets,
                         int32_t* isect_edge_ranges, int64_t num_intersects, void* stream) {
  if (num_intersects < 0) return CS_ERR_ARG;
  if (num_intersects == 0) return CS_OK;
  edge_ranges_kernel<<<ceil_div(num_intersects, 256), 256, 0, (cudaStream_t)stream>>>(
      prim_ids_sorted, prim_edge_offsets, isect_edge_ranges, num_intersects);
  return launch_status();
}

size_t cs_bin_workspace_size(int64_t num_tiles) { return bin_ws_size(num_tiles); }

size_t cs_unit_lists_size(int64_t num_tiles) {
  const long long units = (long long)kStrips * (num_tiles > 0 ? num_tiles : 1);
  return sizeof(int32_t) * (size_t)(kUnitBuckets + kUnitBuckets * units);
}

int cs_bin_count(const float* cubics_norm, const int32_t* prim_seg_offsets, const float* aa_widths,
                 const float* stroke_widths, const float* basis, float* cubics_px,
                 float* edges_px, const int32_t* prim_edge_offsets,
                 int32_t* prim_edge_offsets_out, int32_t* prim_tile_ranges,
                 int32_t* num_tiles_hit, int32_t* tile_bins, int32_t* tile_dlist,
                 int32_t* counters, void* workspace,
                 int64_t num_primitives, int64_t num_segments, int64_t isect_capacity,
                 int64_t dlist_capacity, int32_t samples, int32_t img_height, int32_t img_width,
                 int32_t tile_row_begin, int32_t tile_row_end, float aabb_pad, int32_t aniso,
                 const float* ring, int32_t ring_segs_per_path, void* stream) {
  if (num_primitives < 0 || samples < 2 || img_height <= 0 || img_width <= 0 || !workspace ||
      !counters || !tile_bins || !tile_dlist || (!ring && !cubics_norm) ||
      (ring && (ring_segs_per_path <= 0 || num_segments != num_primitives * ring_segs_per_path)))
    return CS_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int tbx = (img_width + kTile - 1) / kTile, tby = (img_height + kTile - 1) / kTile;
  const long long nt = (long long)tbx * tby;
  const int r0 = max(0, tile_row_begin), r1 = min(tby, tile_row_end);
  BinWorkspace ws = bin_ws(workspace, nt);
  // one launch: a warp per primitive, then the last CTA scans the tile counts
  // (at least one CTA, so that an empty scene still gets empty tile ranges)
  bin_prep_kernel<<<max(1, ceil_div(num_primitives * 32, kPrepThreads)), kPrepThreads, 0, st>>>(
      cubics_norm, ring, ring_segs_per_path, prim_seg_offsets, prim_edge_offsets,
      prim_edge_offsets ? nullptr : prim_edge_offsets_out, aa_widths, stroke_widths, basis,
      cubics_px, edges_px, prim_tile_ranges, num_tiles_hit, ws, tile_bins, tile_dlist, counters,
      num_primitives, num_segments, samples, 0.5f * (float)img_width, 0.5f * (float)img_height,
      tbx, tby, r0, r1, aabb_pad, aniso, (isect_capacity > 0 ? isect_capacity : 0),
      (dlist_capacity > 0 ? dlist_capacity : 0));
  return launch_status();
}

static StageIO stage_io(const int32_t* pids, const float* edges_px, const int32_t* ranges,
                        const int32_t* eoffs, const float* colors, const float* opacities,
                        const float* inv_sigma2s, const int32_t* fill_rules,
                        const float* stroke_widths, int32_t* tile_dlist, void* imeta,
                        int32_t* rowoff, int32_t* istrip, void* dlist, int tbx) {
  StageIO io;
  io.pids = pids;
  io.edges = reinterpret_cast<const float4*>(edges_px);
  io.ranges = reinterpret_cast<const int2*>(ranges);
  io.eoffs = eoffs;
  io.colors = colors;
  io.opac = opacities;
  io.inv_s2 = inv_sigma2s;
  io.rules = fill_rules;
  io.sw = stroke_widths;
  io.dlr = reinterpret_cast<int2*>(tile_dlist);
  io.imeta = reinterpret_cast<IMeta*>(imeta);
  io.rowoff = rowoff;
  io.istrip = reinterpret_cast<int2*>(istrip);
  io.dl = reinterpret_cast<DEntry*>(dlist);
  io.tbx = tbx;
  return io;
}

int cs_bin_sort(const int32_t* prim_tile_ranges, const float* depths, const int32_t* tile_bins,
                int32_t* prim_ids_sorted, int64_t* isect_ids_sorted, int32_t* counters,
                void* workspace, int64_t num_primitives, int64_t isect_capacity,
                int32_t img_height, int32_t img_width, int32_t tile_row_begin,
                int32_t tile_row_end, const float* edges_px, const int32_t* prim_edge_offsets,
                const float* colors, const float* opacities, const float* inv_sigma2s,
                const int32_t* fill_rules, const float* stroke_widths, int32_t* tile_dlist,
                void* imeta, int32_t* rowoff, int32_t* isect_strips, void* dlist,
                int64_t dlist_capacity, int32_t* unit_order, void* stream) {
  if (num_primitives < 0 || isect_capacity < 0 || !workspace || !isect_ids_sorted || !counters)
    return CS_ERR_ARG;
  const bool stage = imeta != nullptr;
  if (stage && (!edges_px || !prim_edge_offsets || !colors || !opacities || !inv_sigma2s ||
                !tile_dlist || !dlist || !isect_strips ||
                (!stroke_widths && (!fill_rules || !rowoff))))
    return CS_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int tbx = (img_width + kTile - 1) / kTile, tby = (img_height + kTile - 1) / kTile;
  const long long nt = (long long)tbx * tby;
  const int r0 = max(0, tile_row_begin), r1 = min(tby, tile_row_end);
  if (r1 <= r0 || num_primitives == 0 || isect_capacity == 0) return CS_OK;
  BinWorkspace ws = bin_ws(workspace, nt);
  unsigned long long* pairs = reinterpret_cast<unsigned long long*>(isect_ids_sorted);
  bin_scatter_kernel<<<ceil_div(num_primitives * 32, 256), 256, 0, st>>>(
      prim_tile_ranges, depths, ws.cursor, pairs, counters, num_primitives, tbx, isect_capacity,
      r0, r1, stage ? unit_order : nullptr);
  StageIO io = stage_io(prim_ids_sorted, edges_px, nullptr, prim_edge_offsets, colors, opacities,
                        inv_sigma2s, fill_rules, stroke_widths, tile_dlist, imeta, rowoff,
                        isect_strips, dlist, tbx);
  dim3 grid(tbx, r1 - r0);
  int* lists = stage ? unit_order : nullptr;  // counts cleared by bin_scatter_kernel
  if (stroke_widths)
    bin_tile_kernel<true><<<grid, kSortThreads, 0, st>>>(
        tile_bins, depths, pairs, prim_ids_sorted, reinterpret_cast<long long*>(isect_ids_sorted),
        counters, isect_capacity, (dlist_capacity > 0 ? dlist_capacity : 0), r0, io, lists);
  else
    bin_tile_kernel<false><<<grid, kSortThreads, 0, st>>>(
        tile_bins, depths, pairs, prim_ids_sorted, reinterpret_cast<long long*>(isect_ids_sorted),
        counters, isect_capacity, (dlist_capacity > 0 ? dlist_capacity : 0), r0, io, lists);
  return launch_status();
}

size_t cs_stage_workspace_size(int64_t num_tiles) { return align256(sizeof(int) * num_tiles); }

int cs_tile_stage(const int32_t* prim_ids_sorted, const int32_t* tile_bins, const float* edges_px,
                  const int32_t* isect_edge_ranges, const int32_t* prim_edge_offsets,
                  const float* colors, const float* opacities, const float* inv_sigma2s,
                  const int32_t* fill_rules, const float* stroke_widths, int32_t* tile_dlist,
                  void* imeta, int32_t* rowoff, int32_t* isect_strips, void* dlist,
                  int32_t* unit_order, int32_t* counters, void* workspace,
                  int64_t dlist_capacity, int32_t img_height, int32_t img_width, void* stream) {
  if (!prim_ids_sorted || !tile_bins || !edges_px || (!isect_edge_ranges && !prim_edge_offsets) ||
      !colors || !opacities || !inv_sigma2s || !tile_dlist || !imeta || !dlist || !counters ||
      !isect_strips ||
      !workspace || (!stroke_widths && (!fill_rules || !rowoff)) || img_height <= 0 ||
      img_width <= 0)
    return CS_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int tbx = (img_width + kTile - 1) / kTile, tby = (img_height + kTile - 1) / kTile;
  const long long nt = (long long)tbx * tby;
  int* ecounts = static_cast<int*>(workspace);
  if (unit_order) cudaMemsetAsync(unit_order, 0, sizeof(int) * kUnitBuckets, st);
  tile_esum_kernel<<<ceil_div(nt * 32, 256), 256, 0, st>>>(
      tile_bins, prim_ids_sorted, reinterpret_cast<const int2*>(isect_edge_ranges),
      prim_edge_offsets, ecounts, nt);
  bin_scan_kernel<<<1, 1024, 0, st>>>(nullptr, ecounts, nullptr, tile_dlist, nullptr, counters,
                                      0, nt, 0, (dlist_capacity > 0 ? dlist_capacity : 0));
  StageIO io = stage_io(prim_ids_sorted, edges_px, isect_edge_ranges, prim_edge_offsets, colors,
                        opacities, inv_sigma2s, fill_rules, stroke_widths, tile_dlist, imeta,
                        rowoff, isect_strips, dlist, tbx);
  dim3 grid(tbx, tby);
  const long long dcap = dlist_capacity > 0 ? dlist_capacity : 0;
  if (stroke_widths)
    tile_stage_kernel<true><<<grid, kSortThreads, 0, st>>>(tile_bins, counters, dcap, io,
                                                           unit_order);
  else
    tile_stage_kernel<false><<<grid, kSortThreads, 0, st>>>(tile_bins, counters, dcap, io,
                                                            unit_order);
  return launch_status();
}

}  // extern "C"
