// Adaptive de Casteljau flattening of pixel-space cubics into straight edges
// with CSR offsets, and the matching edge-gradient accumulation (sm_100a).
//
// The reference splits breadth-first: at each depth every active cubic is
// tested for flatness (control points within tol of the chord) and the
// non-flat ones are split at t = 1/2 into two halves; at the maximum depth
// ceil(log2(S - 1)) every remaining cubic is a leaf.  The leaves are then
// sorted by (segment, t0) (manbo/ops/cubic_splatting.py:1729-1832, with
// cubic_adaptive_flatness_flags :1863-1957 and cubic_split_half :1960-2068).
// Here one thread walks one segment's subdivision tree depth-first, left half
// first: it forms exactly the same child cubics with the same arithmetic and
// meets the leaves already in (segment, t0) order, so no sort is needed.  One
// pass counts each segment's leaves, a scan turns the counts into the CSR
// offsets (segment and primitive), and a second walk writes the leaves.
#include "cs_common.cuh"

namespace cs {

constexpr int kMaxFlattenDepth = 16;  // S - 1 <= 65536 edges per segment

// max / clamp with NaN propagation, as torch.maximum / torch.clamp on the
// reference's host path (the flatness test's written form).
__device__ __forceinline__ float nmax(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return fmaxf(a, b);
}

__device__ __forceinline__ float nclamp_min(float a, float lo) { return a != a ? a : fmaxf(a, lo); }

// Largest distance of the inner control points from the chord (or, for a
// chord of squared length <= 1e-6, the largest distance from the first
// point), compared with tol (cubic_splatting.py:1925-1953).
__device__ __forceinline__ bool cubic_is_flat(const float c[8], float tol) {
  const float eps = 1e-6f;
  const float lx = c[6] - c[0], ly = c[7] - c[1];
  const float chord2 = lx * lx + ly * ly;
  const float v1x = c[2] - c[0], v1y = c[3] - c[1];
  const float v2x = c[4] - c[0], v2y = c[5] - c[1];
  float dmax;
  if (chord2 <= eps) {
    const float n1 = sqrtf(nclamp_min(v1x * v1x + v1y * v1y, 0.0f));
    const float n2 = sqrtf(nclamp_min(v2x * v2x + v2y * v2y, 0.0f));
    const float n3 = sqrtf(nclamp_min(chord2, 0.0f));
    dmax = nmax(n1, nmax(n2, n3));
  } else {
    const float chord = sqrtf(nclamp_min(chord2, eps));
    const float cross1 = fabsf(lx * v1y - ly * v1x);
    const float cross2 = fabsf(lx * v2y - ly * v2x);
    dmax = nmax(cross1 / chord, cross2 / chord);
  }
  return dmax <= tol;
}

// Midpoint subdivision at t = 1/2 (cubic_splatting.py:2000-2028).
__device__ __forceinline__ void cubic_split_half(const float c[8], float l[8], float r[8]) {
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    const float p0 = c[a], p1 = c[2 + a], p2 = c[4 + a], p3 = c[6 + a];
    const float p01 = 0.5f * (p0 + p1), p12 = 0.5f * (p1 + p2), p23 = 0.5f * (p2 + p3);
    const float p012 = 0.5f * (p01 + p12), p123 = 0.5f * (p12 + p23);
    const float p0123 = 0.5f * (p012 + p123);
    l[a] = p0; l[2 + a] = p01; l[4 + a] = p012; l[6 + a] = p0123;
    r[a] = p0123; r[2 + a] = p123; r[4 + a] = p23; r[6 + a] = p3;
  }
}

// Walks segment `seg`'s subdivision tree depth-first, left first.  Counts the
// leaves, and when `out` is given writes leaf j as edge out + j (endpoints
// c[0], c[3]) with its parameter interval.
__device__ int flatten_segment(const float* __restrict__ cubics, long long seg, int maxd,
                               float tol, float4* __restrict__ out, float* __restrict__ t0o,
                               float* __restrict__ t1o) {
  float st[kMaxFlattenDepth + 2][8];
  float sa[kMaxFlattenDepth + 2], sb[kMaxFlattenDepth + 2];
  int sd[kMaxFlattenDepth + 2];
  const float4* src = reinterpret_cast<const float4*>(cubics + seg * 8);
  const float4 q0 = src[0], q1 = src[1];
  st[0][0] = q0.x; st[0][1] = q0.y; st[0][2] = q0.z; st[0][3] = q0.w;
  st[0][4] = q1.x; st[0][5] = q1.y; st[0][6] = q1.z; st[0][7] = q1.w;
  sa[0] = 0.0f;
  sb[0] = 1.0f;
  sd[0] = 0;
  int top = 1, n = 0;
  while (top > 0) {
    --top;
    float c[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) c[k] = st[top][k];
    const float ta = sa[top], tb = sb[top];
    const int d = sd[top];
    if (d >= maxd || cubic_is_flat(c, tol)) {
      if (out) {
        out[n] = make_float4(c[0], c[1], c[6], c[7]);
        t0o[n] = ta;
        t1o[n] = tb;
      }
      ++n;
      continue;
    }
    float l[8], r[8];
    cubic_split_half(c, l, r);
    const float tm = 0.5f * (ta + tb);
    // right half below the left one: the left half is walked first
#pragma unroll
    for (int k = 0; k < 8; ++k) st[top][k] = r[k];
    sa[top] = tm;
    sb[top] = tb;
    sd[top] = d + 1;
#pragma unroll
    for (int k = 0; k < 8; ++k) st[top + 1][k] = l[k];
    sa[top + 1] = ta;
    sb[top + 1] = tm;
    sd[top + 1] = d + 1;
    top += 2;
  }
  return n;
}

__global__ void dc_count_kernel(const float* __restrict__ cubics, int* __restrict__ counts,
                                long long nseg, int maxd, float tol) {
  const long long seg = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (seg >= nseg) return;
  counts[seg + 1] = flatten_segment(cubics, seg, maxd, tol, nullptr, nullptr, nullptr);
}

// One CTA: in-place inclusive scan of offs[1..nseg] (offs[0] = 0), then the
// primitive offsets prim[p] = offs[seg_offs[p]].  Reports CS_ERR_CAPACITY if
// the total exceeds cap and CS_ERR_ARG for segment offsets out of range.
__global__ void __launch_bounds__(1024) dc_scan_kernel(int* __restrict__ offs, long long nseg,
                                                       const int* __restrict__ seg_offs,
                                                       int* __restrict__ prim, long long np,
                                                       long long cap, int* __restrict__ status) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) {
    carry = 0;
    offs[0] = 0;
  }
  __syncthreads();
  for (long long base = 1; base <= nseg; base += 1024) {
    const long long i = base + tid;
    int v = i <= nseg ? offs[i] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane == 31) warp_tot[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int w = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += u;
      }
      warp_tot[lane] = w;
    }
    __syncthreads();
    const int c = carry;
    if (i <= nseg) offs[i] = c + v + (wid > 0 ? warp_tot[wid - 1] : 0);
    __syncthreads();
    if (tid == 0) carry = c + warp_tot[31];
    __syncthreads();
  }
  if (tid == 0 && (long long)carry > cap && status) atomicExch(status, CS_ERR_CAPACITY);
  if (prim) {
    for (long long p = tid; p <= np; p += 1024) {
      const int s = seg_offs[p];
      if (s < 0 || (long long)s > nseg) {
        if (status) atomicExch(status, CS_ERR_ARG);
        prim[p] = 0;
      } else {
        prim[p] = offs[s];
      }
    }
  }
}

__global__ void dc_write_kernel(const float* __restrict__ cubics, const int* __restrict__ offs,
                                float4* __restrict__ edges, float* __restrict__ t0,
                                float* __restrict__ t1, long long nseg, int maxd, float tol,
                                long long cap) {
  const long long seg = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (seg >= nseg) return;
  const long long e0 = offs[seg];
  if (e0 + (offs[seg + 1] - offs[seg]) > cap) return;  // reported by the scan
  flatten_segment(cubics, seg, maxd, tol, edges + e0, t0 + e0, t1 + e0);
}

// v_P_k = sum_e gs_e B_k(t0_e) + ge_e B_k(t1_e) over the segment's CSR edge
// range, in the reference's order (cubic_splatting.py:2399-2487), then an
// optional per-axis scale (the normalised-space epilogue).
__global__ void edge_grads_csr_kernel(const float4* __restrict__ v_edges,
                                      const float* __restrict__ t_start,
                                      const float* __restrict__ t_end,
                                      const int* __restrict__ offs, float* __restrict__ v_cubics,
                                      long long nseg, float sx, float sy) {
  const long long sid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (sid >= nseg) return;
  float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f, a20 = 0.f, a21 = 0.f, a30 = 0.f, a31 = 0.f;
  for (int e = offs[sid]; e < offs[sid + 1]; ++e) {
    const float t0 = t_start[e], t1 = t_end[e];
    const float o0 = 1.0f - t0, o1 = 1.0f - t1;
    const float o0s = o0 * o0, o1s = o1 * o1, t0s = t0 * t0, t1s = t1 * t1;
    const float b00 = o0s * o0, b01 = 3.0f * o0s * t0, b02 = 3.0f * o0 * t0s, b03 = t0s * t0;
    const float b10 = o1s * o1, b11 = 3.0f * o1s * t1, b12 = 3.0f * o1 * t1s, b13 = t1s * t1;
    const float4 g = v_edges[e];
    a00 = a00 + g.x * b00 + g.z * b10;
    a01 = a01 + g.y * b00 + g.w * b10;
    a10 = a10 + g.x * b01 + g.z * b11;
    a11 = a11 + g.y * b01 + g.w * b11;
    a20 = a20 + g.x * b02 + g.z * b12;
    a21 = a21 + g.y * b02 + g.w * b12;
    a30 = a30 + g.x * b03 + g.z * b13;
    a31 = a31 + g.y * b03 + g.w * b13;
  }
  float4* out = reinterpret_cast<float4*>(v_cubics + sid * 8);
  if (sx == 1.0f && sy == 1.0f) {
    out[0] = make_float4(a00, a01, a10, a11);
    out[1] = make_float4(a20, a21, a30, a31);
  } else {
    out[0] = make_float4(a00 * sx, a01 * sy, a10 * sx, a11 * sy);
    out[1] = make_float4(a20 * sx, a21 * sy, a30 * sx, a31 * sy);
  }
}

__global__ void flatness_flags_kernel(const float* __restrict__ cubics, uint8_t* __restrict__ out,
                                      long long n, float tol, int force) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float c[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) c[k] = cubics[i * 8 + k];
  out[i] = (force || cubic_is_flat(c, tol)) ? 1 : 0;
}

__global__ void split_half_kernel(const float* __restrict__ cubics, float* __restrict__ left,
                                  float* __restrict__ right, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float c[8], l[8], r[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) c[k] = cubics[i * 8 + k];
  cubic_split_half(c, l, r);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    left[i * 8 + k] = l[k];
    right[i * 8 + k] = r[k];
  }
}

inline int flatten_max_depth(int samples) {
  const int e = samples - 1;
  int d = 0;
  while (d < 31 && (1 << d) < e) ++d;
  return d;
}

}  // namespace cs

using namespace cs;

extern "C" {

int32_t cs_de_casteljau_max_depth(int32_t samples) {
  return flatten_max_depth(samples < 2 ? 2 : samples);
}

int64_t cs_de_casteljau_edge_capacity(int64_t num_segments, int32_t samples) {
  const int d = flatten_max_depth(samples < 2 ? 2 : samples);
  if (num_segments <= 0 || d > kMaxFlattenDepth) return 0;
  return num_segments << d;
}

int cs_flatten_de_casteljau(const float* cubics_px, const int32_t* prim_seg_offsets,
                            int64_t num_segments, int64_t num_primitives, int32_t samples,
                            float tol_px, float* edges_px, int32_t* prim_edge_offsets,
                            int32_t* segment_edge_offsets, float* edge_t_starts,
                            float* edge_t_ends, int64_t edge_capacity, int32_t* status,
                            void* stream) {
  if (num_segments < 0 || num_primitives < 0 || !segment_edge_offsets ||
      (num_segments > 0 && (!cubics_px || !edges_px || !edge_t_starts || !edge_t_ends)) ||
      (prim_edge_offsets && !prim_seg_offsets))
    return CS_ERR_ARG;
  const int s = samples < 2 ? 2 : samples;
  const int maxd = flatten_max_depth(s);
  if (maxd > kMaxFlattenDepth) return CS_ERR_UNSUPPORTED;
  if (num_segments > 0 && edge_capacity < (num_segments << maxd)) return CS_ERR_CAPACITY;
  if (num_segments + 1 > (int64_t)INT32_MAX || (num_segments << maxd) > (int64_t)INT32_MAX)
    return CS_ERR_UNSUPPORTED;
  const float tol = fmaxf(1e-4f, tol_px);  // the reference's floor (:1731)
  cudaStream_t st = (cudaStream_t)stream;
  if (num_segments > 0)
    dc_count_kernel<<<ceil_div(num_segments, 128), 128, 0, st>>>(cubics_px, segment_edge_offsets,
                                                                num_segments, maxd, tol);
  dc_scan_kernel<<<1, 1024, 0, st>>>(segment_edge_offsets, num_segments, prim_seg_offsets,
                                     prim_edge_offsets, num_primitives, edge_capacity, status);
  if (num_segments > 0)
    dc_write_kernel<<<ceil_div(num_segments, 128), 128, 0, st>>>(
        cubics_px, segment_edge_offsets, reinterpret_cast<float4*>(edges_px), edge_t_starts,
        edge_t_ends, num_segments, maxd, tol, edge_capacity);
  return launch_status();
}

int cs_cubic_flatness_flags(const float* cubics, uint8_t* out_flat, int64_t num_cubics,
                             float tol_px, int32_t force_flat, void* stream) {
  if (num_cubics < 0 || (num_cubics > 0 && (!cubics || !out_flat))) return CS_ERR_ARG;
  if (num_cubics == 0) return CS_OK;
  flatness_flags_kernel<<<ceil_div(num_cubics, 256), 256, 0, (cudaStream_t)stream>>>(
      cubics, out_flat, num_cubics, fmaxf(1e-4f, tol_px), force_flat);
  return launch_status();
}

int cs_cubic_split_half(const float* cubics, float* left, float* right, int64_t num_cubics,
                        void* stream) {
  if (num_cubics < 0 || (num_cubics > 0 && (!cubics || !left || !right))) return CS_ERR_ARG;
  if (num_cubics == 0) return CS_OK;
  split_half_kernel<<<ceil_div(num_cubics, 256), 256, 0, (cudaStream_t)stream>>>(cubics, left,
                                                                                 right, num_cubics);
  return launch_status();
}

int cs_edge_grads_to_cubics_csr(const float* v_edges, const float* edge_t_starts,
                                const float* edge_t_ends, const int32_t* segment_edge_offsets,
                                float* v_cubics, int64_t num_segments, float scale_x,
                                float scale_y, void* stream) {
  if (num_segments < 0 || !segment_edge_offsets || (num_segments > 0 && !v_cubics))
    return CS_ERR_ARG;
  if (num_segments == 0) return CS_OK;
  edge_grads_csr_kernel<<<ceil_div(num_segments, 128), 128, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const float4*>(v_edges), edge_t_starts, edge_t_ends, segment_edge_offsets,
      v_cubics, num_segments, scale_x, scale_y);
  return launch_status();
}

}  // extern "C"
