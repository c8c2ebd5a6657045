// Per-tile staging records shared by the binning kernels (writers) and the
// raster kernels (readers).
//
// For every tile, the edges of its intersects are classified once per frame
// against the tile's pixel-centre box (see raster.cu for why this is exact):
//   * near edges become 32-byte DEntry records, compacted in (intersect, edge)
//     order into one contiguous per-tile range of the D-list, so a raster CTA
//     brings a whole tile's geometry into shared memory with one bulk copy;
//   * far edges that cross tile rows while lying entirely right of the tile
//     become per-row winding offsets (fill mode);
//   * all other edges are dropped.
// Each intersect also gets a 48-byte IMeta record with its primitive's
// colour, opacity, softness and culling distance.
#pragma once

#include <math_constants.h>

#include "cs_common.cuh"

namespace cs {

struct __align__(16) DEntry {
  float4 a;  // x0, y0, vx = x1 - x0, vy = y1 - y0
  float4 b;  // 1 / max(vx^2 + vy^2, eps), y1, x0 * vy, edge id (int bits)
};

struct __align__(16) IMeta {
  int dstart;  // first DEntry of this intersect, relative to the tile's range
  int dcount;  // number of DEntry records
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

}  // namespace cs
