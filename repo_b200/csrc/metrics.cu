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
  // four float4 pairs per thread and round, all loads issued before any use,
  // so each thread keeps 128 bytes in flight
  long long i = t;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 a[4], b[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      a[u] = __ldg(x4 + i + u * stride);
      b[u] = __ldg(y4 + i + u * stride);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float d0 = a[u].x - b[u].x, d1 = a[u].y - b[u].y, d2 = a[u].z - b[u].z,
                  d3 = a[u].w - b[u].w;
      acc = __fmaf_rn(d0, d0, acc);
      acc = __fmaf_rn(d1, d1, acc);
      acc = __fmaf_rn(d2, d2, acc);
      acc = __fmaf_rn(d3, d3, acc);
    }
  }
  for (; i < n4; i += stride) {
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
                                    const float* __restrict__ scale, float factor,
                                    float* __restrict__ grad, long long n) {
  const float s = scale ? *scale * factor : factor;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    grad[i] = s * (lhs[i] - rhs[i]);
}

// --------------------------------------------------------------------------
// SSIM: one launch.  Each CTA computes a 32x32 block of the SSIM map of one
// plane: the (32+R)^2 input window is loaded to shared memory, a horizontal
// pass writes the five windowed moments (x, y, x^2, y^2, xy) for 32 output
// columns, each thread producing 8 columns of one input row, then a vertical
// pass produces 4 output rows of one column per thread.  Both passes walk
// their inputs once and scatter each into the outputs whose window covers it,
// so every product is formed once and every sum still adds its taps in
// window order.  The window size is a template parameter, so no tap is
// predicated away.  Per-CTA SSIM sums are reduced per plane by the last CTA
// to finish.

constexpr int kSsimT = 32;         // output tile edge
constexpr int kSsimThreads = 256;
constexpr int kMaxWin = 15;

template <int WIN>
__global__ void __launch_bounds__(kSsimThreads, 4) ssim_kernel(
    const float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ gauss,
    int h, int w, float c1, float c2, float inv_count, float* __restrict__ ssim_map,
    float* __restrict__ partials, unsigned int* __restrict__ ticket,
    float* __restrict__ plane_means) {
  constexpr int R = WIN - 1;
  constexpr int IN = kSsimT + R;  // even, so the pitch IN + 1 is odd
  constexpr int LOADS = (IN * IN + kSsimThreads - 1) / kSsimThreads;
  __shared__ float sx[IN][IN + 1];
  __shared__ float sy[IN][IN + 1];
  __shared__ float2 hp[2][IN][kSsimT + 1];  // (mu_x, mu_y), (E[x^2], E[y^2]) per row
  __shared__ float h4[IN][kSsimT + 1];       // E[xy]
  __shared__ float g[WIN];
  __shared__ float red[kSsimThreads / 32];
  __shared__ bool last;
  const long long plane = blockIdx.z;
  const int oh = h - R, ow = w - R;
  const int ox0 = blockIdx.x * kSsimT, oy0 = blockIdx.y * kSsimT;
  const float* xp = x + plane * (long long)h * w;
  const float* yp = y + plane * (long long)h * w;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid < WIN) g[tid] = gauss[tid];
  {
    // all of a thread's loads are issued before any is stored, so the tile
    // costs one memory round trip rather than one per element
    float xa[LOADS], ya[LOADS];
#pragma unroll
    for (int i = 0; i < LOADS; ++i) {
      const int idx = tid + i * kSsimThreads;
      const int r = idx / IN, c = idx - r * IN;
      const int gy = oy0 + r, gx = ox0 + c;
      const bool ok = idx < IN * IN && gy < h && gx < w;
      xa[i] = ok ? __ldg(xp + (long long)gy * w + gx) : 0.0f;
      ya[i] = ok ? __ldg(yp + (long long)gy * w + gx) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < LOADS; ++i) {
      const int idx = tid + i * kSsimThreads;
      if (idx < IN * IN) {
        const int r = idx / IN, c = idx - r * IN;
        sx[r][c] = xa[i];
        sy[r][c] = ya[i];
      }
    }
  }
  __syncthreads();
  float gk[WIN];
#pragma unroll
  for (int k = 0; k < WIN; ++k) gk[k] = g[k];
  // horizontal: (input row r, output columns c0 .. c0+7).  Warps 0-3 take rows
  // 0-31 of column group `wid` (lanes = rows: distinct banks); warps 4-5 take
  // the remaining R rows of all four groups.
  {
    int r = lane, grp = wid;
    bool active = wid < 4;
    if (R > 0 && wid >= 4) {
      const int j = tid - 128;
      grp = j / (R > 0 ? R : 1);
      r = 32 + (j - grp * (R > 0 ? R : 1));
      active = j < 4 * R;
    }
    if (active) {
      // (mu_x, mu_y) and (E[x^2], E[y^2]) share their weights: packed FP32x2
      // multiply-adds, each component rounded as the scalar one
      const int c0 = grp * 8;
      float2 m12[8], e1122[8];
      float e12[8];
#pragma unroll
      for (int o = 0; o < 8; ++o) {
        m12[o] = e1122[o] = make_float2(0.0f, 0.0f);
        e12[o] = 0.0f;
      }
#pragma unroll
      for (int q = 0; q < 8 + R; ++q) {
        const float2 uv2 = make_float2(sx[r][c0 + q], sy[r][c0 + q]);
        const float2 sq = __fmul2_rn(uv2, uv2);
        const float uv = uv2.x * uv2.y;
#pragma unroll
        for (int o = 0; o < 8; ++o) {
          const int k = q - o;
          if (k >= 0 && k < WIN) {
            const float2 gg = make_float2(gk[k], gk[k]);
            m12[o] = __ffma2_rn(gg, uv2, m12[o]);
            e1122[o] = __ffma2_rn(gg, sq, e1122[o]);
            e12[o] = __fmaf_rn(gk[k], uv, e12[o]);
          }
        }
      }
#pragma unroll
      for (int o = 0; o < 8; ++o) {
        hp[0][r][c0 + o] = m12[o];
        hp[1][r][c0 + o] = e1122[o];
        h4[r][c0 + o] = e12[o];
      }
    }
  }
  __syncthreads();
  // vertical: (output column lane, output rows r0 .. r0+3)
  float local = 0.0f;
  {
    const int c = lane, r0 = wid * 4;
    float mom[4][5];
#pragma unroll
    for (int q = 0; q < 2; ++q) {  // the moment pairs, packed
      float2 acc[4];
#pragma unroll
      for (int o = 0; o < 4; ++o) acc[o] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int t = 0; t < 4 + R; ++t) {
        const float2 val = hp[q][r0 + t][c];
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          const int k = t - o;
          if (k >= 0 && k < WIN) acc[o] = __ffma2_rn(make_float2(gk[k], gk[k]), val, acc[o]);
        }
      }
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        mom[o][2 * q] = acc[o].x;
        mom[o][2 * q + 1] = acc[o].y;
      }
    }
    {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int t = 0; t < 4 + R; ++t) {
        const float val = h4[r0 + t][c];
#pragma unroll
        for (int o = 0; o < 4; ++o) {
          const int k = t - o;
          if (k >= 0 && k < WIN) acc[o] = __fmaf_rn(gk[k], val, acc[o]);
        }
      }
#pragma unroll
      for (int o = 0; o < 4; ++o) mom[o][4] = acc[o];
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

// Launch the instance for an odd window size 1 <= win <= kMaxWin.
inline void launch_ssim(int win, dim3 grid, cudaStream_t st, const float* x, const float* y,
                        const float* gauss, int h, int w, float c1, float c2, float inv_count,
                        float* ssim_map, float* partials, unsigned int* ticket,
                        float* plane_means) {
#define CS_SSIM_CASE(WIN)                                                                  \
  case WIN:                                                                                \
    ssim_kernel<WIN><<<grid, kSsimThreads, 0, st>>>(x, y, gauss, h, w, c1, c2, inv_count,  \
                                                    ssim_map, partials, ticket, plane_means); \
    break;
  switch (win) {
    CS_SSIM_CASE(1)
    CS_SSIM_CASE(3)
    CS_SSIM_CASE(5)
    CS_SSIM_CASE(7)
    CS_SSIM_CASE(9)
    CS_SSIM_CASE(11)
    CS_SSIM_CASE(13)
    CS_SSIM_CASE(15)
    default:
      break;
  }
#undef CS_SSIM_CASE
}

// Fixed scratch of cs_ssim_noalloc: one copy per device, loaded with the
// module.  Bytes [0, 256) hold the completion ticket, the partial sums follow.
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) unsigned char
    g_ssim_noalloc_scratch[256 + sizeof(float) * CS_SSIM_NOALLOC_MAX_PARTIALS];
static std::atomic<unsigned char*> g_ssim_noalloc_base[kNoAllocMaxDevices];

inline int mse_blocks(long long n) {
  long long b = (n + kMseThreads * 16 - 1) / (kMseThreads * 16);  // 16 elements per thread
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

int cs_mse_backward(const float* lhs, const float* rhs, const float* scale, float factor,
                    float* grad, int64_t n, void* stream) {
  if (n < 0) return CS_ERR_ARG;
  if (n == 0) return CS_OK;
  int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
  mse_backward_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(lhs, rhs, scale, factor, grad, n);
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
  launch_ssim(win, dim3(gx, gy, (unsigned)planes), st, x, y, gauss, h, w, c1, c2, inv_count,
              ssim_map, partials, ticket, plane_means);
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
  launch_ssim(win, dim3(gx, gy, (unsigned)planes), st, x, y, gauss, h, w, c1, c2, inv_count,
              ssim_map, partials, ticket, plane_means);
  return launch_status();
}

}  // extern "C"
