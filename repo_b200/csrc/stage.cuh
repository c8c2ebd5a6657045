// Per-tile staging records shared by the binning kernels (writers) and the
// raster kernels (readers).
//
// A 16x16 tile is rasterised as kStrips strips of kStripRows pixel rows, one
// warp per strip.  For every tile, the edges of its intersects are classified
// once per frame against each strip's pixel-centre box (see raster.cu for why
// this is exact):
//   * an edge within the primitive's culling distance of a strip becomes a
//     32-byte DEntry record in that strip's list; each strip's list is
//     compacted in (intersect, edge) order into its own contiguous range of
//     the D-list, so a raster warp brings its strip's geometry into shared
//     memory with bulk copies;
//   * far edges that cross tile rows while lying entirely right of the tile
//     become per-row winding offsets (fill mode);
//   * all other edges are dropped.
// Each intersect also gets a 48-byte IMeta record with its primitive's
// colour, opacity, softness and culling distance, and per strip the range
// (first record, record count) of its records in the strip's list.
#pragma once

#include <math_constants.h>

#include "cs_common.cuh"

namespace cs {

struct __align__(16) DEntry {
  float4 a;  // x0, y0, vx = x1 - x0, vy = y1 - y0
  float4 b;  // 1 / max(vx^2 + vy^2, eps), y1, x0 * vy, edge id (int bits)
};

constexpr int kStrips = 4;                  // strips per tile
constexpr int kStripRows = kTile / kStrips;  // pixel rows per strip (one warp: 4 x 16 px)

struct __align__(16) IMeta {
  int dstart;  // unused (0): per-strip ranges are kept beside the records
  int dcount;  // unused (0)
  int pid;     // primitive id
  int rule;    // fill rule (0 even-odd, else nonzero); 1 for strokes
  float c0, c1, c2, op;
  float a;     // fill: sqrt(max(1/sigma^2, eps)); stroke: max(1/sigma^2, eps)
  float b;     // stroke: half stroke width; fill: 0
  float dthr;  // culling distance (pixels); +inf disables culling
  float spare;
};

// Row winding offsets are packed per row: low 16 bits signed winding sum,
// high 16 bits crossing count (parity = count & 1).
__device__ __forceinline__ int pack_row(int wind, int cnt) {
  return (wind & 0xffff) | (cnt << 16);
}
__device__ __forceinline__ int row_wind(int packed) { return (int)(short)(packed & 0xffff); }
__device__ __forceinline__ int row_cnt(int packed) { return (int)((unsigned)packed >> 16); }

// Distance beyond which a pixel's coverage is saturated for this primitive.
// Fill: inside, logit <= -20 gives exp(logit) < 2^-25 so 1/(1+exp) == 1.0f
// exactly; outside, logit >= ln(255 op) + 1 keeps op*cov below 1/(255 e).
// Stroke: 1/2 edge_d^2 / sigma^2 >= ln(255 op) + 1 keeps op*cov below alpha_min.
// Half a pixel of margin covers rounding of the distance itself.
template <bool STROKE>
__device__ __forceinline__ void intersect_attrs(int pid, const float* __restrict__ colors,
                                                const float* __restrict__ opac,
                                                const float* __restrict__ inv_s2,
                                                const int* __restrict__ rules,
                                                const float* __restrict__ sw, IMeta& m) {
  m.pid = pid;
  m.c0 = colors[pid * 3];
  m.c1 = colors[pid * 3 + 1];
  m.c2 = colors[pid * 3 + 2];
  const float op = opac[pid];
  m.op = op;
  const float is2 = inv_s2[pid];
  const float lg = logf(fmaxf(255.0f * op, 1.0f)) + 1.0f;
  if (!STROKE) {
    m.a = sqrtf(fmaxf(is2, kEps));
    m.b = 0.0f;
    m.rule = rules[pid];
    const float L = fmaxf(20.0f, lg);
    m.dthr = (L <= 59.0f && m.a > 0.0f) ? 0.5f * L / m.a + 0.5f : CUDART_INF_F;
  } else {
    m.a = fmaxf(is2, kEps);
    m.b = fmaxf(0.0f, sw[pid]) * 0.5f;
    m.rule = 1;
    m.dthr = m.b + sqrtf(2.0f * lg / m.a) + 0.5f;
  }
  if (!(m.dthr == m.dthr)) m.dthr = CUDART_INF_F;
  m.spare = 0.0f;
}

// Edge within d of the pixel-centre box [bx0, bx0+15] x [by0, by0+15]
// (bounding-box test, conservative).  Non-finite or very large coordinates
// are always treated as near so that the exact per-pixel path handles them.
__device__ __forceinline__ bool edge_is_near(const float4& e, float d, float bx0, float by0) {
  const float bx1 = bx0 + 15.0f, by1 = by0 + 15.0f;
  const bool moderate = fabsf(e.x) < 4.0e6f && fabsf(e.y) < 4.0e6f && fabsf(e.z) < 4.0e6f &&
                        fabsf(e.w) < 4.0e6f;
  const float xmin = fminf(e.x, e.z), xmax = fmaxf(e.x, e.z);
  const float ymin = fminf(e.y, e.w), ymax = fmaxf(e.y, e.w);
  return !moderate ||
         (xmax >= bx0 - d && xmin <= bx1 + d && ymax >= by0 - d && ymin <= by1 + d);
}

// Bit s set when the edge comes within d of strip s's pixel-centre box
// [bx0, bx0+15] x [by0 + 4s, by0 + 4s + 3]; the union over strips is
// edge_is_near for the whole tile.
__device__ __forceinline__ unsigned edge_near_strips(const float4& e, float d, float bx0,
                                                     float by0) {
  const float bx1 = bx0 + 15.0f;
  const bool moderate = fabsf(e.x) < 4.0e6f && fabsf(e.y) < 4.0e6f && fabsf(e.z) < 4.0e6f &&
                        fabsf(e.w) < 4.0e6f;
  if (!moderate) return (1u << kStrips) - 1u;
  const float xmin = fminf(e.x, e.z), xmax = fmaxf(e.x, e.z);
  if (!(xmax >= bx0 - d && xmin <= bx1 + d)) return 0u;
  const float ymin = fminf(e.y, e.w), ymax = fmaxf(e.y, e.w);
  unsigned m = 0u;
#pragma unroll
  for (int st = 0; st < kStrips; ++st) {
    const float sy0 = by0 + (float)(st * kStripRows), sy1 = sy0 + (float)(kStripRows - 1);
    if (ymax >= sy0 - d && ymin <= sy1 + d) m |= 1u << st;
  }
  return m;
}

// Rows (bits of a 16-bit tile row mask) of the strips in strip mask m.
__device__ __forceinline__ unsigned strip_rows(unsigned m) {
  unsigned r = 0u;
#pragma unroll
  for (int st = 0; st < kStrips; ++st)
    if (m & (1u << st)) r |= ((1u << kStripRows) - 1u) << (st * kStripRows);
  return r;
}

// Far edge entirely right of the box that spans some of its rows: it crosses
// every pixel of row r when y0 <= py < y1 or y1 <= py < y0 (py = by0 + r), far
// beyond rounding error of the reference's crossing test.
__device__ __forceinline__ unsigned far_right_rows(const float4& e, float bx0, float by0) {
  const float bx1 = bx0 + 15.0f, by1 = by0 + 15.0f;
  if (!(fminf(e.x, e.z) > bx1) || fmaxf(e.y, e.w) < by0 || fminf(e.y, e.w) > by1) return 0u;
  unsigned rows = 0u;
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    const float py = by0 + (float)r;
    if (((e.y <= py) & (e.w > py)) | ((e.y > py) & (e.w <= py))) rows |= 1u << r;
  }
  return rows;
}

__device__ __forceinline__ DEntry make_entry(const float4& e, int eid) {
  const float vx = e.z - e.x, vy = e.w - e.y;
  const float vv = vx * vx + vy * vy;
  DEntry d;
  d.a = make_float4(e.x, e.y, vx, vy);
  d.b = make_float4(1.0f / fmaxf(vv, kEps), e.w, e.x * vy, __int_as_float(eid));
  return d;
}

// Dispatch lists of raster work units ("unit lists"): int32 [kUnitBuckets +
// kUnitBuckets * nunits]: the count of every work bucket, then one list of
// capacity nunits per bucket.  The staging pass appends every unit to the
// bucket of its work estimate (two buckets per octave, heaviest first, no
// work last); the raster kernels take units bucket by bucket.  The order
// within a bucket is arbitrary: it affects scheduling only.
constexpr int kUnitBuckets = 64;

__device__ __forceinline__ int work_bucket(int w) {
  if (w <= 0) return kUnitBuckets - 1;
  const int msb = 31 - __clz(w);
  const int half = msb >= 1 ? (w >> (msb - 1)) & 1 : 0;
  return (kUnitBuckets - 2) - min(2 * msb + half, kUnitBuckets - 2);
}

__device__ __forceinline__ void append_unit(int* lists, int nunits, int unit, int weight) {
  const int b = work_bucket(weight);
  const int pos = atomicAdd(lists + b, 1);
  lists[kUnitBuckets + (long long)b * nunits + pos] = unit;
}

// Unit at dispatch position u (u < nunits), for a warp whose lane l holds the
// exclusive prefix counts pre0 = start of bucket 2l and pre1 = start of 2l+1.
__device__ __forceinline__ int unit_at(const int* lists, int nunits, int u, int pre0, int pre1) {
  const unsigned q = __ballot_sync(0xffffffffu, pre0 <= u);  // bit 0 is always set
  const int L = 31 - __clz(q);
  const int p0 = __shfl_sync(0xffffffffu, pre0, L), p1 = __shfl_sync(0xffffffffu, pre1, L);
  const int b = 2 * L + (p1 <= u ? 1 : 0);
  const int base = p1 <= u ? p1 : p0;
  return __ldg(lists + kUnitBuckets + (long long)b * nunits + (u - base));
}

// Per-lane bucket starts for unit_at (one warp).
__device__ __forceinline__ void unit_prefix(const int* lists, int& pre0, int& pre1) {
  const int lane = threadIdx.x & 31;
  const int c0 = __ldg(lists + 2 * lane), c1 = __ldg(lists + 2 * lane + 1);
  const int pair = c0 + c1;
  const int incl = warp_incl_scan(pair, lane);
  pre0 = incl - pair;
  pre1 = pre0 + c0;
}

}  // namespace cs
