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
#include <atomic>

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
// SSIM: one launch.  Each CTA computes a 32x32 block of the SSIM map of one
// plane: the (32+R)^2 input window is loaded to shared memory, a horizontal
// pass writes the five windowed moments (x, y, x^2, y^2, xy) for 32 output
// columns, each thread producing 8 columns from one register window, then a
// vertical pass produces 4 output rows per thread the same way.  Per-CTA SSIM
// sums are reduced per plane by the last CTA to finish.

constexpr int kSsimT = 32;         // output tile edge
constexpr int kSsimThreads = 256;
constexpr int kMaxWin = 15;
constexpr int kMaxR = kMaxWin - 1;
constexpr int kSsimIn = kSsimT + kMaxR;

__global__ void __launch_bounds__(kSsimThreads) ssim_kernel(
    const float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ gauss,
    int h, int w, int win, float c1, float c2, float inv_count, float* __restrict__ ssim_map,
    float* __restrict__ partials, unsigned int* __restrict__ ticket,
    float* __restrict__ plane_means) {
  __shared__ float sx[kSsimIn][kSsimIn + 1];
  __shared__ float sy[kSsimIn][kSsimIn + 1];
  __shared__ float hs[5][kSsimIn][kSsimT + 1];
  __shared__ float g[kMaxWin];
  __shared__ float red[kSsimThreads / 32];
  __shared__ bool last;
  const int R = win - 1;
  const int in_n = kSsimT + R;
  const long long plane = blockIdx.z;
  const int oh = h - R, ow = w - R;
  const int ox0 = blockIdx.x * kSsimT, oy0 = blockIdx.y * kSsimT;
  const float* xp = x + plane * (long long)h * w;
  const float* yp = y + plane * (long long)h * w;
  const int tid = threadIdx.x;
  if (tid < win) g[tid] = gauss[tid];
  for (int idx = tid; idx < in_n * in_n; idx += kSsimThreads) {
    const int r = idx / in_n, c = idx - r * in_n;
    const int gy = oy0 + r, gx = ox0 + c;
    const bool ok = gy < h && gx < w;
    sx[r][c] = ok ? __ldg(xp + (long long)gy * w + gx) : 0.0f;
    sy[r][c] = ok ? __ldg(yp + (long long)gy * w + gx) : 0.0f;
  }
  __syncthreads();
  // horizontal: item = (input row r, 8 output columns)
  for (int item = tid; item < in_n * (kSsimT / 8); item += kSsimThreads) {
    const int r = item >> 2, c0 = (item & 3) * 8;
    float a[8 + kMaxR], b[8 + kMaxR];
#pragma unroll
    for (int q = 0; q < 8 + kMaxR; ++q) {
      a[q] = q < 8 + R ? sx[r][c0 + q] : 0.0f;
      b[q] = q < 8 + R ? sy[r][c0 + q] : 0.0f;
    }
#pragma unroll
    for (int o = 0; o < 8; ++o) {
      float m1 = 0.f, m2 = 0.f, e11 = 0.f, e22 = 0.f, e12 = 0.f;
#pragma unroll
      for (int k = 0; k < kMaxWin; ++k) {
        if (k < win) {
          const float gk = g[k], u = a[o + k], v = b[o + k];
          m1 = __fmaf_rn(gk, u, m1);
          m2 = __fmaf_rn(gk, v, m2);
          e11 = __fmaf_rn(gk, u * u, e11);
          e22 = __fmaf_rn(gk, v * v, e22);
          e12 = __fmaf_rn(gk, u * v, e12);
        }
      }
      hs[0][r][c0 + o] = m1;
      hs[1][r][c0 + o] = m2;
      hs[2][r][c0 + o] = e11;
      hs[3][r][c0 + o] = e22;
      hs[4][r][c0 + o] = e12;
    }
  }
  __syncthreads();
  // vertical: item = (output column c, 4 output rows)
  float local = 0.0f;
  {
    const int c = tid & 31, r0 = (tid >> 5) * 4;
    float mom[4][5];
#pragma unroll
    for (int o = 0; o < 4; ++o)
#pragma unroll
      for (int q = 0; q < 5; ++q) mom[o][q] = 0.0f;
#pragma unroll
    for (int q = 0; q < 5; ++q) {
      float col[4 + kMaxR];
#pragma unroll
      for (int t = 0; t < 4 + kMaxR; ++t) col[t] = t < 4 + R ? hs[q][r0 + t][c] : 0.0f;
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < kMaxWin; ++k)
          if (k < win) acc = __fmaf_rn(g[k], col[o + k], acc);
        mom[o][q] = acc;
      }
    }
#pragma unroll
    for (int o = 0; o < 4; ++o) {
      const int oy = oy0 + r0 + o, ox = ox0 + c;
      if (oy >= oh || ox >= ow) continue;
      const float mu1 = mom[o][0], mu2 = mom[o][1];
      const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu12 = mu1 * mu2;
      const float s1 = mom[o][2] - mu1_sq, s2 = mom[o][3] - mu2_sq, s12 = mom[o][4] - mu12;
      const float lum = (2.0f * mu12 + c1) / (mu1_sq + mu2_sq + c1);
      const float cs_ = (2.0f * s12 + c2) / (s1 + s2 + c2);
      const float v = lum * cs_;
      if (ssim_map) ssim_map[(plane * oh + oy) * (long long)ow + ox] = v;
      local += v;
    }
  }
  const float bs = block_sum(local, red);
  const unsigned tiles = gridDim.x * gridDim.y;
  const unsigned nblk = tiles * gridDim.z;
  if (tid == 0) {
    partials[plane * tiles + blockIdx.y * gridDim.x + blockIdx.x] = bs;
    __threadfence();
    last = atomicAdd(ticket, 1u) == nblk - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (unsigned pl = 0; pl < gridDim.z; ++pl) {
    float v = 0.0f;
    for (unsigned q = tid; q < tiles; q += kSsimThreads) v += partials[pl * tiles + q];
    const float t = block_sum(v, red);
    if (tid == 0) plane_means[pl] = t * inv_count;
  }
  if (tid == 0) *ticket = 0u;
}

// Fixed scratch of cs_ssim_noalloc: one copy per device, loaded with the
// module.  Bytes [0, 256) hold the completion ticket, the partial sums follow.
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) unsigned char
    g_ssim_noalloc_scratch[256 + sizeof(float) * CS_SSIM_NOALLOC_MAX_PARTIALS];
static std::atomic<unsigned char*> g_ssim_noalloc_base[kNoAllocMaxDevices];

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
  gx = (w - win + 1 + kSsimT - 1) / kSsimT;
  gy = (h - win + 1 + kSsimT - 1) / kSsimT;
}

size_t cs_ssim_workspace_size(int64_t planes, int32_t h, int32_t w, int32_t win) {
  int gx, gy;
  ssim_grid(h, w, win, gx, gy);
  return 256 + sizeof(float) * (size_t)planes * gx * gy;
}

int cs_ssim(const float* x, const float* y, const float* gauss, int64_t planes, int32_t h,
            int32_t w, int32_t win, float c1, float c2, float* plane_means, float* ssim_map,
            void* workspace, void* stream) {
  if (planes <= 0 || win <= 0 || win % 2 == 0 || h < win || w < win || !workspace ||
      !plane_means)
    return CS_ERR_ARG;
  if (win > kMaxWin || planes > 65535) return CS_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  int gx, gy;
  ssim_grid(h, w, win, gx, gy);
  const int R = win - 1;
  unsigned int* ticket = static_cast<unsigned int*>(workspace);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  const float inv_count = 1.0f / ((float)(h - R) * (float)(w - R));
  ssim_kernel<<<dim3(gx, gy, (unsigned)planes), kSsimThreads, 0, st>>>(
      x, y, gauss, h, w, win, c1, c2, inv_count, ssim_map, partials, ticket, plane_means);
  return launch_status();
}

int cs_ssim_noalloc(const float* x, const float* y, const float* gauss, int64_t planes,
                    int32_t h, int32_t w, int32_t win, float c1, float c2, float* plane_means,
                    float* ssim_map, void* stream) {
  if (planes <= 0 || win <= 0 || win % 2 == 0 || h < win || w < win || !plane_means)
    return CS_ERR_ARG;
  if (win > kMaxWin || planes > 65535) return CS_ERR_UNSUPPORTED;
  int gx, gy;
  ssim_grid(h, w, win, gx, gy);
  if (planes * (int64_t)gx * gy > CS_SSIM_NOALLOC_MAX_PARTIALS) return CS_ERR_CAPACITY;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return CS_ERR_CUDA;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return CS_ERR_UNSUPPORTED;
  unsigned char* base = g_ssim_noalloc_base[dev].load(std::memory_order_acquire);
  if (!base) {
    // The symbol's address differs per device; it is resolved with `dev`
    // current.  Two threads racing here store the same value.
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_ssim_noalloc_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return CS_ERR_CUDA;
    }
    base = static_cast<unsigned char*>(p);
    g_ssim_noalloc_base[dev].store(base, std::memory_order_release);
  }
  cudaStream_t st = (cudaStream_t)stream;
  unsigned int* ticket = reinterpret_cast<unsigned int*>(base);
  float* partials = reinterpret_cast<float*>(base + 256);
  if (cudaMemsetAsync(ticket, 0, sizeof(unsigned int), st) != cudaSuccess) {
    cudaGetLastError();
    return CS_ERR_CUDA;
  }
  const int R = win - 1;
  const float inv_count = 1.0f / ((float)(h - R) * (float)(w - R));
  ssim_kernel<<<dim3(gx, gy, (unsigned)planes), kSsimThreads, 0, st>>>(
      x, y, gauss, h, w, win, c1, c2, inv_count, ssim_map, partials, ticket, plane_means);
  return launch_status();
}

}  // extern "C"
