// Image metrics: MSE / SSE, the MSE gradient and SSIM (sm_100a).
//
// These kernels are HBM-bound streaming reductions.  The MSE forward is one
// launch: grid-stride float4 loads, warp + CTA reduction into per-CTA
// partials, and the last CTA to finish (atomic ticket) sums the partials in a
// fixed order, so the result is deterministic and needs no host loop
// (the reference launches mse_partial_sum_kernel and then
// reduce_sum_partial_kernel until one value is left, manbo/ops/metric.py:344-382).
// SSIM uses the separability of the Gaussian window: a horizontal 11-tap pass
// into shared memory, then a vertical pass, instead of the reference's direct
// 121-tap window (manbo/ops/metric.py:300-339).
#include <algorithm>

#include "cs_common.cuh"

namespace cs {

constexpr int kMseThreads = 256;
constexpr int kMseMaxBlocks = 148 * 8;

__device__ __forceinline__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  float r = 0.0f;
  if (wid == 0) {
    r = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0.0f;
    r = warp_sum(r);
  }
  __syncthreads();
  return r;  // valid in warp 0
}

__global__ void __launch_bounds__(kMseThreads) mse_kernel(const float* __restrict__ x,
                                                          const float* __restrict__ y, long long n,
                                                          float* __restrict__ partials,
                                                          unsigned int* __restrict__ counter,
                                                          float* __restrict__ out_sse,
                                                          float* __restrict__ out_mse) {
  __shared__ float sh[32];
  __shared__ bool last;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  float acc = 0.0f;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  long long n4 = vec ? n / 4 : 0;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const float4* y4 = reinterpret_cast<const float4*>(y);
  for (long long i = t; i < n4; i += stride) {
    float4 a = x4[i], b = y4[i];
    float d0 = a.x - b.x, d1 = a.y - b.y, d2 = a.z - b.z, d3 = a.w - b.w;
    acc = __fmaf_rn(d0, d0, acc);
    acc = __fmaf_rn(d1, d1, acc);
    acc = __fmaf_rn(d2, d2, acc);
    acc = __fmaf_rn(d3, d3, acc);
  }
  for (long long i = n4 * 4 + t; i < n; i += stride) {
    float d = x[i] - y[i];
    acc = __fmaf_rn(d, d, acc);
  }
  float bs = block_sum(acc, sh);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = bs;
    __threadfence();
    unsigned int ticket = atomicAdd(counter, 1u);
    last = ticket == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float v = 0.0f;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) v += partials[i];
  float total = block_sum(v, sh);
  if (threadIdx.x == 0) {
    if (out_sse) *out_sse = total;
    if (out_mse) *out_mse = total / (float)n;
    *counter = 0u;
  }
}

__global__ void mse_backward_kernel(const float* __restrict__ lhs, const float* __restrict__ rhs,
                                    const float* __restrict__ scale, float* __restrict__ grad,
                                    long long n) {
  const float s = *scale;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    grad[i] = s * (lhs[i] - rhs[i]);
}

// --------------------------------------------------------------------------
// SSIM

constexpr int kSsimTx = 32;   // output tile width
constexpr int kSsimTy = 16;   // output tile height
constexpr int kSsimThreads = 256;
constexpr int kMaxWin = 15;

__global__ void __launch_bounds__(kSsimThreads) ssim_tile_kernel(
    const float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ gauss,
    int h, int w, int win, float c1, float c2, float* __restrict__ ssim_map,
    float* __restrict__ partials) {
  extern __shared__ float smem[];
  const int R = win - 1;
  const int in_w = kSsimTx + R, in_h = kSsimTy + R;
  float* sx = smem;                          // [in_h][in_w]
  float* sy = sx + in_h * in_w;
  float* hs = sy + in_h * in_w;              // 5 x [in_h][kSsimTx]
  __shared__ float g[kMaxWin];
  __shared__ float red[32];
  const long long plane = blockIdx.z;
  const int oh = h - R, ow = w - R;
  const int ox0 = blockIdx.x * kSsimTx, oy0 = blockIdx.y * kSsimTy;
  const float* xp = x + plane * (long long)h * w;
  const float* yp = y + plane * (long long)h * w;
  if (threadIdx.x < win) g[threadIdx.x] = gauss[threadIdx.x];
  for (int idx = threadIdx.x; idx < in_h * in_w; idx += kSsimThreads) {
    int r = idx / in_w, c = idx - r * in_w;
    int gy = oy0 + r, gx = ox0 + c;
    bool ok = gy < h && gx < w;
    sx[idx] = ok ? xp[(long long)gy * w + gx] : 0.0f;
    sy[idx] = ok ? yp[(long long)gy * w + gx] : 0.0f;
  }
  __syncthreads();
  const int plane_sz = in_h * kSsimTx;
  for (int idx = threadIdx.x; idx < plane_sz; idx += kSsimThreads) {
    int r = idx / kSsimTx, c = idx - r * kSsimTx;
    float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
    const float* rx = sx + r * in_w + c;
    const float* ry = sy + r * in_w + c;
    for (int k = 0; k < win; ++k) {
      float gk = g[k], a = rx[k], b = ry[k];
      m1 = __fmaf_rn(gk, a, m1);
      m2 = __fmaf_rn(gk, b, m2);
      e11 = __fmaf_rn(gk, a * a, e11);
      e22 = __fmaf_rn(gk, b * b, e22);
      e12 = __fmaf_rn(gk, a * b, e12);
    }
    hs[idx] = m1;
    hs[plane_sz + idx] = m2;
    hs[2 * plane_sz + idx] = e11;
    hs[3 * plane_sz + idx] = e22;
    hs[4 * plane_sz + idx] = e12;
  }
  __syncthreads();
  float local = 0.0f;
  for (int idx = threadIdx.x; idx < kSsimTx * kSsimTy; idx += kSsimThreads) {
    int r = idx / kSsimTx, c = idx - r * kSsimTx;
    int oy = oy0 + r, ox = ox0 + c;
    if (oy >= oh || ox >= ow) continue;
    float mu1 = 0.f, mu2 = 0.f, ex2 = 0.f, ey2 = 0.f, exy = 0.f;
    for (int k = 0; k < win; ++k) {
      int o = (r + k) * kSsimTx + c;
      float gk = g[k];
      mu1 = __fmaf_rn(gk, hs[o], mu1);
      mu2 = __fmaf_rn(gk, hs[plane_sz + o], mu2);
      ex2 = __fmaf_rn(gk, hs[2 * plane_sz + o], ex2);
      ey2 = __fmaf_rn(gk, hs[3 * plane_sz + o], ey2);
      exy = __fmaf_rn(gk, hs[4 * plane_sz + o], exy);
    }
    float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu12 = mu1 * mu2;
    float s1 = ex2 - mu1_sq, s2 = ey2 - mu2_sq, s12 = exy - mu12;
    float lum = (2.0f * mu12 + c1) / (mu1_sq + mu2_sq + c1);
    float cs_ = (2.0f * s12 + c2) / (s1 + s2 + c2);
    float v = lum * cs_;
    if (ssim_map) ssim_map[(plane * oh + oy) * (long long)ow + ox] = v;
    local += v;
  }
  float bs = block_sum(local, red);
  if (threadIdx.x == 0)
    partials[plane * (long long)(gridDim.x * gridDim.y) + blockIdx.y * gridDim.x + blockIdx.x] = bs;
}

__global__ void ssim_reduce_kernel(const float* __restrict__ partials, int nblk, float inv_count,
                                   float* __restrict__ plane_means) {
  __shared__ float red[32];
  const long long plane = blockIdx.x;
  float v = 0.0f;
  for (int i = threadIdx.x; i < nblk; i += blockDim.x) v += partials[plane * nblk + i];
  float t = block_sum(v, red);
  if (threadIdx.x == 0) plane_means[plane] = t * inv_count;
}

inline int mse_blocks(long long n) {
  long long b = (n + kMseThreads * 8 - 1) / (kMseThreads * 8);
  return (int)std::max<long long>(1, std::min<long long>(b, kMseMaxBlocks));
}

}  // namespace cs

using namespace cs;

extern "C" {

size_t cs_mse_workspace_size(int64_t n) {
  (void)n;
  return 256 + sizeof(float) * kMseMaxBlocks;
}

int cs_mse_forward(const float* x, const float* y, int64_t n, float* out_sse, float* out_mse,
                   void* workspace, void* stream) {
  if (n <= 0 || !x || !y || !workspace) return CS_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned int* counter = static_cast<unsigned int*>(workspace);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  cudaMemsetAsync(counter, 0, sizeof(unsigned int), st);
  mse_kernel<<<mse_blocks(n), kMseThreads, 0, st>>>(x, y, n, partials, counter, out_sse, out_mse);
  return launch_status();
}

int cs_mse_backward(const float* lhs, const float* rhs, const float* scale, float* grad, int64_t n,
                    void* stream) {
  if (n < 0 || !scale) return CS_ERR_ARG;
  if (n == 0) return CS_OK;
  int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
  mse_backward_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(lhs, rhs, scale, grad, n);
  return launch_status();
}

static inline void ssim_grid(int32_t h, int32_t w, int32_t win, int& gx, int& gy) {
  gx = (w - win + 1 + kSsimTx - 1) / kSsimTx;
  gy = (h - win + 1 + kSsimTy - 1) / kSsimTy;
}

size_t cs_ssim_workspace_size(int64_t planes, int32_t h, int32_t w, int32_t win) {
  int gx, gy;
  ssim_grid(h, w, win, gx, gy);
  return sizeof(float) * (size_t)planes * gx * gy;
}

int cs_ssim(const float* x, const float* y, const float* gauss, int64_t planes, int32_t h,
            int32_t w, int32_t win, float c1, float c2, float* plane_means, float* ssim_map,
            void* workspace, void* stream) {
  if (planes <= 0 || win <= 0 || win % 2 == 0 || win > kMaxWin || h < win || w < win ||
      !workspace || !plane_means)
    return CS_ERR_ARG;
  if (planes > 65535) return CS_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  int gx, gy;
  ssim_grid(h, w, win, gx, gy);
  const int R = win - 1;
  size_t smem = sizeof(float) * ((size_t)2 * (kSsimTy + R) * (kSsimTx + R) +
                                 (size_t)5 * (kSsimTy + R) * kSsimTx);
  float* partials = static_cast<float*>(workspace);
  ssim_tile_kernel<<<dim3(gx, gy, (unsigned)planes), kSsimThreads, smem, st>>>(
      x, y, gauss, h, w, win, c1, c2, ssim_map, partials);
  float inv_count = 1.0f / ((float)(h - R) * (float)(w - R));
  ssim_reduce_kernel<<<(unsigned)planes, 256, 0, st>>>(partials, gx * gy, inv_count, plane_means);
  return launch_status();
}

}  // extern "C"
