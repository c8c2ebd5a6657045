// Adan optimiser step (sm_100a): the update of manbo/ops/optim.py:29-106
// (adan_step_from_grad_kernel), element by element, in one HBM-streaming pass.
//
// Per element: reads param, grad, exp_avg, exp_avg_sq, exp_avg_diff,
// neg_pre_grad (24 B), writes all but grad (20 B).  The kernel is bandwidth
// bound; it moves four elements per thread with 16-byte accesses when every
// buffer is 16-byte aligned and falls back to single elements otherwise.
// Arithmetic is the reference's, in its written order, in float32.
#include <algorithm>

#include "cs_common.cuh"

namespace cs {

struct AdanArgs {
  float b1, b2, b3, bc1, bc2, bc3s, lr, wd, eps, clip;
  int first;    // step == 1: the gradient difference starts at zero
  int no_prox;  // decoupled (true) or proximal (false) weight decay
};

__device__ __forceinline__ void adan_one(const AdanArgs& a, float& p, float g_raw, float& m,
                                         float& n, float& d, float& npg) {
  const float g = g_raw * a.clip;
  const float ngod = a.first ? 0.0f : npg + g;  // g_t - g_{t-1}
  const float m_t = m * a.b1 + g * (1.0f - a.b1);
  const float d_t = d * a.b2 + ngod * (1.0f - a.b2);
  const float ngod2 = ngod * a.b2 + g;
  const float n_t = n * a.b3 + ngod2 * ngod2 * (1.0f - a.b3);
  const float denom = sqrtf(n_t) / a.bc3s + a.eps;
  const float step_size = a.lr / a.bc1;
  const float step_size_diff = a.lr * a.b2 / a.bc2;
  float q = p;
  if (a.no_prox) {
    q = q * (1.0f - a.lr * a.wd);
    q = q - step_size * m_t / denom;
    q = q - step_size_diff * d_t / denom;
  } else {
    q = q - step_size * m_t / denom;
    q = q - step_size_diff * d_t / denom;
    q = q / (1.0f + a.lr * a.wd);
  }
  p = q;
  m = m_t;
  d = d_t;
  n = n_t;
  npg = -g;
}

__global__ void adan_kernel4(float4* __restrict__ p, const float4* __restrict__ g,
                             float4* __restrict__ m, float4* __restrict__ n,
                             float4* __restrict__ d, float4* __restrict__ npg, long long n4,
                             AdanArgs a) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 P = p[i], M = m[i], N = n[i], D = d[i], Q = npg[i];
    const float4 G = __ldg(g + i);
    adan_one(a, P.x, G.x, M.x, N.x, D.x, Q.x);
    adan_one(a, P.y, G.y, M.y, N.y, D.y, Q.y);
    adan_one(a, P.z, G.z, M.z, N.z, D.z, Q.z);
    adan_one(a, P.w, G.w, M.w, N.w, D.w, Q.w);
    p[i] = P;
    m[i] = M;
    n[i] = N;
    d[i] = D;
    npg[i] = Q;
  }
}

__global__ void adan_kernel1(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ n, float* __restrict__ d,
                             float* __restrict__ npg, long long count, AdanArgs a) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
    float P = p[i], M = m[i], N = n[i], D = d[i], Q = npg[i];
    adan_one(a, P, __ldg(g + i), M, N, D, Q);
    p[i] = P;
    m[i] = M;
    n[i] = N;
    d[i] = D;
    npg[i] = Q;
  }
}

inline bool aligned16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace cs

using namespace cs;

extern "C" {

int cs_adan_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq,
                 float* exp_avg_diff, float* neg_pre_grad, int64_t numel, int32_t step,
                 float beta1, float beta2, float beta3, float bias_correction1,
                 float bias_correction2, float bias_correction3_sqrt, float lr,
                 float weight_decay, float eps, float clip_global_grad_norm, int32_t no_prox,
                 void* stream) {
  if (numel < 0 || step < 1) return CS_ERR_ARG;
  if (numel == 0) return CS_OK;
  if (!param || !grad || !exp_avg || !exp_avg_sq || !exp_avg_diff || !neg_pre_grad)
    return CS_ERR_ARG;
  AdanArgs a;
  a.b1 = beta1;
  a.b2 = beta2;
  a.b3 = beta3;
  a.bc1 = bias_correction1;
  a.bc2 = bias_correction2;
  a.bc3s = bias_correction3_sqrt;
  a.lr = lr;
  a.wd = weight_decay;
  a.eps = eps;
  a.clip = clip_global_grad_norm;
  a.first = step == 1;
  a.no_prox = no_prox != 0;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = numel % 4 == 0 && aligned16(param) && aligned16(grad) && aligned16(exp_avg) &&
                   aligned16(exp_avg_sq) && aligned16(exp_avg_diff) && aligned16(neg_pre_grad);
  const long long items = vec ? numel / 4 : numel;
  const int blocks = (int)std::min<long long>((items + 255) / 256, 148LL * 8);
  if (vec)
    adan_kernel4<<<blocks, 256, 0, st>>>(
        reinterpret_cast<float4*>(param), reinterpret_cast<const float4*>(grad),
        reinterpret_cast<float4*>(exp_avg), reinterpret_cast<float4*>(exp_avg_sq),
        reinterpret_cast<float4*>(exp_avg_diff), reinterpret_cast<float4*>(neg_pre_grad), items,
        a);
  else
    adan_kernel1<<<blocks, 256, 0, st>>>(param, grad, exp_avg, exp_avg_sq, exp_avg_diff,
                                         neg_pre_grad, items, a);
  return launch_status();
}

}  // extern "C"
