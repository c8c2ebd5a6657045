// Cubic-domain kernels: edge-gradient accumulation onto cubic control points
// and the closed control-polygon -> ring-of-cubics conversion (sm_100a).
#include <algorithm>

#include "cs_common.cuh"

namespace cs {

// v_P_k = sum_e gs_e B_k(e/E) + ge_e B_k((e+1)/E), in the reference's
// summation order (manbo/ops/cubic_splatting.py:2338-2394), then an optional
// per-axis scale (the normalised-space epilogue, :3096-3100).
__global__ void edge_grads_kernel(const float4* __restrict__ v_edges, float* __restrict__ v_cubics,
                                  long long nseg, int E, float sx, float sy) {
  long long sid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (sid >= nseg) return;
  const float inv_e = 1.0f / (float)E;
  float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f, a20 = 0.f, a21 = 0.f, a30 = 0.f, a31 = 0.f;
  for (int e = 0; e < E; ++e) {
    float t0 = (float)e * inv_e, t1 = (float)(e + 1) * inv_e;
    float o0 = 1.0f - t0, o1 = 1.0f - t1;
    float o0s = o0 * o0, o1s = o1 * o1, t0s = t0 * t0, t1s = t1 * t1;
    float b00 = o0s * o0, b01 = 3.0f * o0s * t0, b02 = 3.0f * o0 * t0s, b03 = t0s * t0;
    float b10 = o1s * o1, b11 = 3.0f * o1s * t1, b12 = 3.0f * o1 * t1s, b13 = t1s * t1;
    float4 g = v_edges[sid * E + e];
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

// Anti-aliasing widths -> clamped widths and 1/sigma^2 (the renderer's
// prologue, cubic_splatting.py:2820-2821): w = clamp(aa, min=1e-4),
// inv = 1 / clamp(w * w, min=1e-6), NaN propagating like torch.clamp.
__global__ void aa_widths_forward_kernel(const float* __restrict__ aa, float* __restrict__ w_out,
                                         float* __restrict__ inv_out, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float a = aa[i];
  const float w = a != a ? a : fmaxf(a, 1e-4f);
  const float w2 = w * w;
  const float d = w2 != w2 ? w2 : fmaxf(w2, 1e-6f);
  w_out[i] = w;
  inv_out[i] = 1.0f / d;
}

// v_aa = -2 v_inv / clamp(w^3, min=1e-12) with the clamped widths (the
// backward epilogue, cubic_splatting.py:3101-3104), then, given the raw
// widths, the backward of the entry's clamp(aa, min=1e-4): zero where
// !(aa >= 1e-4), as torch's clamp backward.
__global__ void aa_widths_backward_kernel(const float* __restrict__ aa,
                                          const float* __restrict__ w,
                                          const float* __restrict__ v_inv,
                                          float* __restrict__ v_aa, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float wi = w[i];
  const float w3 = wi * wi * wi;
  const float d = w3 != w3 ? w3 : fmaxf(w3, 1e-12f);
  const float g = (-2.0f * v_inv[i]) / d;
  v_aa[i] = (aa && !(aa[i] >= 1e-4f)) ? 0.0f : g;
}

// Closed K-point control polygon -> two degree-(K/2) Bernstein branches ->
// `subdiv` Hermite cubics per branch (manbo/ops/cubic_splatting.py:190-266).
__global__ void ring_forward_kernel(const float* __restrict__ cp, const float* __restrict__ basis,
                                    const float* __restrict__ dbasis, const float* __restrict__ dt,
                                    float* __restrict__ out, long long nseg, int K, int sub) {
  long long sid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (sid >= nseg) return;
  const int kb = (K + 2) / 2, spc = 2 * sub;
  const float degree = (float)(kb - 1), third = (float)(1.0 / 3.0);
  long long curve = sid / spc;
  int local = (int)(sid - curve * spc);
  int branch = local / sub, s = local - branch * sub, sn = s + 1;
  int base = branch * (kb - 1);
  const float* c = cp + curve * K * 2;
  float p0x = 0.f, p0y = 0.f, p3x = 0.f, p3y = 0.f, d0x = 0.f, d0y = 0.f, d1x = 0.f, d1y = 0.f;
  for (int i = 0; i < kb; ++i) {
    int idx = base + i;
    if (idx >= K) idx -= K;
    float w0 = basis[s * kb + i], w1 = basis[sn * kb + i];
    float x = c[2 * idx], y = c[2 * idx + 1];
    p0x = p0x + w0 * x; p0y = p0y + w0 * y;
    p3x = p3x + w1 * x; p3y = p3y + w1 * y;
  }
  for (int i = 0; i < kb - 1; ++i) {
    int ic = base + i, in = ic + 1;
    if (ic >= K) ic -= K;
    if (in >= K) in -= K;
    float dx = c[2 * in] - c[2 * ic], dy = c[2 * in + 1] - c[2 * ic + 1];
    float db0 = dbasis[s * (kb - 1) + i], db1 = dbasis[sn * (kb - 1) + i];
    d0x = d0x + db0 * dx; d0y = d0y + db0 * dy;
    d1x = d1x + db1 * dx; d1y = d1y + db1 * dy;
  }
  d0x = d0x * degree; d0y = d0y * degree; d1x = d1x * degree; d1y = d1y * degree;
  float dts = dt[s] * third;
  float* o = out + sid * 8;
  o[0] = p0x; o[1] = p0y; o[6] = p3x; o[7] = p3y;
  o[2] = p0x + d0x * dts; o[3] = p0y + d0y * dts;
  o[4] = p3x - d1x * dts; o[5] = p3y - d1y * dts;
}

// Adjoint of ring_forward_kernel with atomics into the control points
// (manbo/ops/cubic_splatting.py:321-395).
__global__ void ring_backward_kernel(const float* __restrict__ gseg, const float* __restrict__ basis,
                                     const float* __restrict__ dbasis, const float* __restrict__ dt,
                                     float* __restrict__ gcp, long long nseg, int K, int sub) {
  long long sid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (sid >= nseg) return;
  const int kb = (K + 2) / 2, spc = 2 * sub;
  const float degree = (float)(kb - 1), third = (float)(1.0 / 3.0);
  long long curve = sid / spc;
  int local = (int)(sid - curve * spc);
  int branch = local / sub, s = local - branch * sub, sn = s + 1;
  int base = branch * (kb - 1);
  float dts = dt[s] * third;
  const float* g = gseg + sid * 8;
  float g0x = g[0] + g[2], g0y = g[1] + g[3];
  float g3x = g[6] + g[4], g3y = g[7] + g[5];
  float gd0x = g[2] * dts, gd0y = g[3] * dts;
  float gd1x = -g[4] * dts, gd1y = -g[5] * dts;
  float* gc = gcp + curve * K * 2;
  for (int i = 0; i < kb; ++i) {
    int idx = base + i;
    if (idx >= K) idx -= K;
    float w0 = basis[s * kb + i], w1 = basis[sn * kb + i];
    atomicAdd(gc + 2 * idx, g0x * w0 + g3x * w1);
    atomicAdd(gc + 2 * idx + 1, g0y * w0 + g3y * w1);
  }
  for (int i = 0; i < kb - 1; ++i) {
    int ic = base + i, in = ic + 1;
    if (ic >= K) ic -= K;
    if (in >= K) in -= K;
    float db0 = dbasis[s * (kb - 1) + i], db1 = dbasis[sn * (kb - 1) + i];
    float dcx = degree * (gd0x * db0 + gd1x * db1);
    float dcy = degree * (gd0y * db0 + gd1y * db1);
    atomicAdd(gc + 2 * ic, -dcx);
    atomicAdd(gc + 2 * ic + 1, -dcy);
    atomicAdd(gc + 2 * in, dcx);
    atomicAdd(gc + 2 * in + 1, dcy);
  }
}

// ---------------------------------------------------------------------------
// ring parameterisation of closed paths: ring [P, 3G, 2] pixel-space points,
// segment k of a path = (r[3k], r[3k+1], r[3k+2], r[3k+3 mod 3G])

// cubics_norm = ring point / (W/2, H/2) - 1 (IEEE division, then subtraction)
__global__ void ring_to_cubics_kernel(const float* __restrict__ ring, float* __restrict__ cn,
                                      long long npaths, int G, float half_w, float half_h) {
  const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // control point
  const long long total = npaths * G * 4;
  if (q >= total) return;
  const long long path = q / (4 * G);
  const int local = (int)(q - path * 4 * G);
  const int k = local >> 2, j = local & 3;
  int r = 3 * k + j;
  if (r >= 3 * G) r -= 3 * G;
  const float2 v = reinterpret_cast<const float2*>(ring)[path * 3 * G + r];
  reinterpret_cast<float2*>(cn)[q] = make_float2(v.x / half_w - 1.0f, v.y / half_h - 1.0f);
}

// Edge endpoint gradients -> ring point gradients.  Each segment's control
// point gradient is the reference's Bernstein accumulation scaled to
// normalised space (x W/2, H/2); the ring gradient is that divided by
// (W/2, H/2) (the derivative of the normalisation), summed over the one or
// two control points that share the ring point.  One CTA handles whole
// paths; optionally v_edges is cleared after it is read.
//
// One warp per path (a grid-stride loop over paths): a path whose tile rows
// miss the band [r0, r1) has no edge gradient here and only writes zeros, so
// a band's launch costs little beyond its own paths.  A live path's segments
// go eight at a time to groups of four lanes: lane `sub` of a group takes
// edges sub, sub + 4, ... of its segment (loaded four at a time),
// and the group reduce-scatters its 8 control-point sums in two shuffle
// rounds, after which lane `sub` holds control point sub; the segments' sums
// wait in shared memory for the ring points.
constexpr int kRingThreads = 128;  // 4 warps per CTA
constexpr int kRingMaxSegs = 128;  // segments per path
constexpr int kRingEdgeLanes = 4;  // lanes per segment (one per control point)
constexpr int kRingSegsPerRound = 32 / kRingEdgeLanes;

__global__ void __launch_bounds__(kRingThreads) edge_grads_to_ring_kernel(
    float4* __restrict__ v_edges, float* __restrict__ v_ring, long long npaths, int G, int E,
    float half_w, float half_h, int clear, const int4* __restrict__ prim_ranges, int r0, int r1) {
  __shared__ float cub[kRingThreads / 32][kRingMaxSegs][8];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int sub = lane & (kRingEdgeLanes - 1), sl = lane / kRingEdgeLanes;
  const float inv_e = 1.0f / (float)E;
  float(*sc)[8] = cub[wid];
  const long long nwarps = (long long)gridDim.x * (kRingThreads / 32);
  for (long long p = (long long)blockIdx.x * (kRingThreads / 32) + wid; p < npaths;
       p += nwarps) {
    bool live = true;
    if (prim_ranges) {
      const int4 rr = __ldg(prim_ranges + p);
      live = max(rr.y, r0) < min(rr.w, r1) && rr.x < rr.z;
    }
    float2* out = reinterpret_cast<float2*>(v_ring) + p * 3 * G;
    if (!live) {
      for (int t = lane; t < 3 * G; t += 32) out[t] = make_float2(0.0f, 0.0f);
      continue;
    }
    for (int s0 = 0; s0 < G; s0 += kRingSegsPerRound) {  // uniform trip count over the warp
      const int seg = s0 + sl;
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (seg < G) {
        float4* gseg = v_edges + (p * G + seg) * E;
        // four of the lane's edges per pass, their loads issued together
        for (int e0 = sub; e0 < E; e0 += 4 * kRingEdgeLanes) {
          float4 gv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e = e0 + i * kRingEdgeLanes;
            gv[i] = e < E ? gseg[e] : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e = e0 + i * kRingEdgeLanes;
            if (e >= E) continue;
            if (clear) gseg[e] = make_float4(0.f, 0.f, 0.f, 0.f);
            const float t0 = (float)e * inv_e, t1 = (float)(e + 1) * inv_e;
            const float o0 = 1.0f - t0, o1 = 1.0f - t1;
            const float o0s = o0 * o0, o1s = o1 * o1, t0s = t0 * t0, t1s = t1 * t1;
            const float b0[4] = {o0s * o0, 3.0f * o0s * t0, 3.0f * o0 * t0s, t0s * t0};
            const float b1[4] = {o1s * o1, 3.0f * o1s * t1, 3.0f * o1 * t1s, t1s * t1};
            const float4 g = gv[i];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              a[2 * c] = a[2 * c] + g.x * b0[c] + g.z * b1[c];
              a[2 * c + 1] = a[2 * c + 1] + g.y * b0[c] + g.w * b1[c];
            }
          }
        }
      }
      // reduce-scatter over the group: values 4-7 to lanes with bit 1 set,
      // 0-3 to the others, then one pair per lane: lane sub keeps values
      // 2 sub, 2 sub + 1 (control point sub's x, y)
      const bool hi2 = (sub & 2) != 0, hi1 = (sub & 1) != 0;
      float k4[4], f[2];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float send = hi2 ? a[i] : a[4 + i], keep = hi2 ? a[4 + i] : a[i];
        k4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = hi1 ? k4[i] : k4[2 + i], keep = hi1 ? k4[2 + i] : k4[i];
        f[i] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
      }
      if (seg < G) {
        sc[seg][2 * sub] = (f[0] * half_w) / half_w;
        sc[seg][2 * sub + 1] = (f[1] * half_h) / half_h;
      }
    }
    __syncwarp();
    for (int t = lane; t < 3 * G; t += 32) {
      const int k = t / 3, j = t - 3 * k;
      float gx = sc[k][2 * j], gy = sc[k][2 * j + 1];
      if (j == 0) {  // shared with the end point of the previous segment
        const int sp = k == 0 ? G - 1 : k - 1;
        gx = gx + sc[sp][6];
        gy = gy + sc[sp][7];
      }
      out[t] = make_float2(gx, gy);
    }
    __syncwarp();  // the sums are read before the next path overwrites them
  }
}

// ---------------------------------------------------------------------------
// Adam over one flat parameter buffer with two learning rates (elements
// [0, n_first) use lr0, the rest lr1):  m = b1 m + (1-b1) g,
// v = b2 v + (1-b2) g^2, p -= lr (m / (1-b1^t)) / (sqrt(v / (1-b2^t)) + eps),
// t = *step + 1 read on the device; the last CTA to finish stores t.
// Optionally the gradient is cleared after use.
__global__ void adam_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, long long n, long long n_first, float lr0,
                            float lr1, float b1, float b2, float eps, int* __restrict__ step,
                            unsigned int* __restrict__ ticket, int clear) {
  __shared__ bool last;
  const int t = *step + 1;
  const float bc1 = 1.0f - powf(b1, (float)t);
  const float bc2 = 1.0f - powf(b2, (float)t);
  const float rb2 = 1.0f / sqrtf(bc2);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float pi = p[i], mi = m[i], vi = v[i];
    adam_element(pi, mi, vi, g[i], i < n_first ? lr0 : lr1, b1, b2, eps, bc1, rb2);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (clear) g[i] = 0.0f;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *step = t;
    *ticket = 0u;
  }
}

}  // namespace cs

using namespace cs;

extern "C" {

int cs_edge_grads_to_cubics(const float* v_edges, float* v_cubics, int64_t num_segments,
                            int32_t edges_per_segment, float scale_x, float scale_y,
                            void* stream) {
  if (num_segments < 0 || edges_per_segment <= 0) return CS_ERR_ARG;
  if (num_segments == 0) return CS_OK;
  edge_grads_kernel<<<ceil_div(num_segments, 128), 128, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const float4*>(v_edges), v_cubics, num_segments, edges_per_segment,
      scale_x, scale_y);
  return launch_status();
}

int cs_aa_widths_forward(const float* aa_widths, float* widths_clamped, float* inv_sigma2s,
                         int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!aa_widths || !widths_clamped || !inv_sigma2s))) return CS_ERR_ARG;
  if (n == 0) return CS_OK;
  aa_widths_forward_kernel<<<ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(
      aa_widths, widths_clamped, inv_sigma2s, n);
  return launch_status();
}

int cs_aa_widths_backward(const float* aa_widths, const float* widths_clamped,
                          const float* v_inv_sigma2s, float* v_aa_widths, int64_t n,
                          void* stream) {
  if (n < 0 || (n > 0 && (!widths_clamped || !v_inv_sigma2s || !v_aa_widths))) return CS_ERR_ARG;
  if (n == 0) return CS_OK;
  aa_widths_backward_kernel<<<ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(
      aa_widths, widths_clamped, v_inv_sigma2s, v_aa_widths, n);
  return launch_status();
}

int cs_ring_segments_forward(const float* control_points, const float* basis,
                             const float* deriv_basis, const float* dt, float* segments,
                             int64_t num_curves, int32_t k, int32_t subdiv, void* stream) {
  if (num_curves < 0 || k < 4 || (k - 2) % 2 != 0 || subdiv <= 0) return CS_ERR_ARG;
  long long n = num_curves * 2LL * subdiv;
  if (n == 0) return CS_OK;
  ring_forward_kernel<<<ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(
      control_points, basis, deriv_basis, dt, segments, n, k, subdiv);
  return launch_status();
}

int cs_ring_segments_backward(const float* grad_segments, const float* basis,
                              const float* deriv_basis, const float* dt,
                              float* grad_control_points, int64_t num_curves, int32_t k,
                              int32_t subdiv, void* stream) {
  if (num_curves < 0 || k < 4 || (k - 2) % 2 != 0 || subdiv <= 0) return CS_ERR_ARG;
  long long n = num_curves * 2LL * subdiv;
  if (n == 0) return CS_OK;
  ring_backward_kernel<<<ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(
      grad_segments, basis, deriv_basis, dt, grad_control_points, n, k, subdiv);
  return launch_status();
}

int cs_ring_to_cubics(const float* ring, float* cubics_norm, int64_t num_paths,
                      int32_t segs_per_path, int32_t img_height, int32_t img_width, void* stream) {
  if (num_paths < 0 || segs_per_path <= 0 || img_height <= 0 || img_width <= 0) return CS_ERR_ARG;
  const long long n = num_paths * segs_per_path * 4;
  if (n == 0) return CS_OK;
  ring_to_cubics_kernel<<<ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(
      ring, cubics_norm, num_paths, segs_per_path, 0.5f * (float)img_width,
      0.5f * (float)img_height);
  return launch_status();
}

int cs_edge_grads_to_ring(float* v_edges, float* v_ring, int64_t num_paths, int32_t segs_per_path,
                          int32_t edges_per_segment, int32_t img_height, int32_t img_width,
                          int32_t clear_edges, const int32_t* prim_tile_ranges,
                          int32_t tile_row_begin, int32_t tile_row_end, void* stream) {
  if (num_paths < 0 || segs_per_path <= 0 || segs_per_path > kRingMaxSegs ||
      edges_per_segment <= 0)
    return CS_ERR_ARG;
  if (num_paths == 0) return CS_OK;
  const long long warps = std::min<long long>(num_paths, 148LL * 64);
  edge_grads_to_ring_kernel<<<(int)ceil_div(warps, kRingThreads / 32), kRingThreads, 0,
                              (cudaStream_t)stream>>>(
      reinterpret_cast<float4*>(v_edges), v_ring, num_paths, segs_per_path, edges_per_segment,
      0.5f * (float)img_width, 0.5f * (float)img_height, clear_edges,
      reinterpret_cast<const int4*>(prim_tile_ranges), tile_row_begin, tile_row_end);
  return launch_status();
}

size_t cs_adam_workspace_size(void) { return 256; }

int cs_adam_step(float* params, float* grads, float* exp_avg, float* exp_avg_sq, int64_t n,
                 int64_t n_first, float lr_first, float lr_rest, float beta1, float beta2,
                 float eps, int32_t* step, void* workspace, int32_t clear_grads, void* stream) {
  if (n < 0 || n_first < 0 || !step || !workspace) return CS_ERR_ARG;
  if (n == 0) return CS_OK;
  const int blocks = (int)((n + 255) / 256 < 148 * 4 ? (n + 255) / 256 : 148 * 4);
  adam_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      params, grads, exp_avg, exp_avg_sq, n, n_first, lr_first, lr_rest, beta1, beta2, eps, step,
      static_cast<unsigned int*>(workspace), clear_grads);
  return launch_status();
}

}  // extern "C"
