// Shared device helpers for the CubicSplat sm_100a kernels.
//
// All kernels in this library are compiled with -fmad=false: a floating-point
// expression is evaluated exactly as written, one IEEE rounding per operation,
// so the per-pixel arithmetic reproduces the reference's formulas
// (manbo/ops/cubic_splatting.py) in a fixed, documented order.  Fused
// multiply-adds appear only where written out with __fmaf_rn.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "cubicsplat_b200.h"

namespace cs {

constexpr float kAlphaCap = 0.999f;
constexpr float kAlphaMin = (float)(1.0 / 255.0);
constexpr float kTransStop = 1e-4f;
constexpr float kEps = 1e-6f;
constexpr int kTile = 16;

// exp(x) by Cody-Waite range reduction (x = k ln2 + r, ln2 split into a
// 16-bit high part and a low correction) and the degree-7 Taylor polynomial
// of exp(r) in Horner form with fused multiply-adds; 2^k is built from its
// exponent bits.  Relative error below 1.3 ulp on [-87, 88].  Inputs below
// -87 return 0 so no subnormal is ever produced.
__device__ __forceinline__ float cs_expf(float x) {
  if (x != x) return x;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  if (x < -87.0f) return 0.0f;
  const float log2e = 1.44269504088896341f;
  const float ln2_hi = 0.693145751953125f;
  const float ln2_lo = 1.42860676533018708e-06f;
  float kf = rintf(__fmul_rn(x, log2e));
  float r = __fmaf_rn(kf, -ln2_hi, x);
  r = __fmaf_rn(kf, -ln2_lo, r);
  float p = 1.0f / 5040.0f;
  p = __fmaf_rn(p, r, 1.0f / 720.0f);
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int k = (int)kf;  // k in [-126, 127] on the accepted domain
  return __fmul_rn(p, __int_as_float((k + 127) << 23));
}

// float -> int32 with truncation toward zero, saturation and NaN -> 0
// (cvt.rzi.s32.f32), the semantics of the reference's T.Cast(int32, float).
__device__ __forceinline__ int f2i_trunc_sat(float v) { return __float2int_rz(v); }

// One Adam element (torch.optim.Adam's update with bias corrections bc1 =
// 1 - b1^t and rb2 = 1 / sqrt(1 - b2^t)), in place on p, m, v.
__device__ __forceinline__ void adam_element(float& p, float& m, float& v, float g, float lr,
                                             float b1, float b2, float eps, float bc1,
                                             float rb2) {
  const float mi = b1 * m + (1.0f - b1) * g;
  const float vi = b2 * v + (1.0f - b2) * g * g;
  m = mi;
  v = vi;
  p = p - (lr / bc1) * mi / (sqrtf(vi) * rb2 + eps);
}

__device__ __forceinline__ uint32_t depth_sort_key(float depth) {
  // Integer order of the key equals float order of the depth, for both signs
  // (manbo/ops/cubic_splatting.py:799-805).
  int32_t bits = __float_as_int(depth);
  int32_t mask = (bits >> 31) | (int32_t)0x80000000;
  return (uint32_t)(bits ^ mask);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_min_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ int warp_max_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// inclusive warp prefix sum
__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CS_OK : CS_ERR_CUDA;
}

}  // namespace cs
