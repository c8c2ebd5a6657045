// Regularisation loss of the curve model (sm_100a): one forward launch for
// the whole scalar and one backward launch for all gradients, instead of the
// reference's partial-sum kernel, reduction and host arithmetic per term
// (manbo/regularization.py:65-250, manbo/ops/regularization.py).
//
//   L = lambda_proj / N * sum phi(alpha)                     (shape)
//     + opacity_weight * mean |sigmoid(op) - 1|              (opacity)
//     + [closed] sum masked |prev - 2 curr + next|^2 / (N P) (curvature)
//     + [closed] sum hinge(joint coordinates) / (N J 2)      (boundary)
//
// phi(a) = relu(a - 1)^2 + relu(-a)^2 with a = ((m - p0) . v) / (|v|^2 + 1e-8),
// v = pend - p0, over each curve's middle control points m (open: pend =
// p[K-1]; closed: pend = p[split], which is skipped), :32-54 and :119-295.
// Curvature samples f = 0, s, 2s, ... of the closed path [xyz[:, 0], reversed
// xyz[:, 1]] (length L = 2M, P = ceil(L / s)) with prev/next 5 samples
// back/ahead, kept where the cosine of the angle at the sample exceeds
// cos(thresh) (:423-515, :646-699).  Joints are p[0], p[d], p[2d], ...
// (J = ceil(K / d)), :357-420.
//
// Every term of every kind is one index of a single grid-stride loop; each
// thread adds its weighted terms, CTAs write partial sums and the last CTA to
// finish adds them in a fixed order (double) into the loss.  The backward
// uses the reference's per-term gradients and scales (:702-1237), with the
// incoming gradient (a device scalar) folded into the scales.

#include "cs_common.cuh"

namespace cs {

struct RegArgs {
  const float* cp;   // [N, K, 2]
  const float* op;   // [n_op]
  const float* xyz;  // [N, 2, M, 2] (closed only)
  long long n, k, n_op, m;
  int closed, split, bdeg, stride;
  float bound, cos_thresh;
  float w_shape, w_op, w_curv, w_bound;  // per-term weights of the loss
  long long t_shape, t_op, t_bound, t_curv;
  long long joints, per_curve;
};

constexpr int kRegThreads = 256;
constexpr int kRegRoll = 5;

// Geometry of shape term t: curve c, its middle point and chord end, v =
// pend - p0, u = mid - p0 and |v|^2 + 1e-8.
__device__ __forceinline__ void shape_geometry(const RegArgs& a, long long t, long long& c,
                                               int& mid, int& pend, float& vx, float& vy,
                                               float& ux, float& uy, float& denom) {
  const long long mc = a.k - 2;
  c = t / mc;
  const int j = (int)(t - c * mc) + 1;
  pend = a.closed ? a.split : (int)a.k - 1;
  mid = a.closed && j >= a.split ? j + 1 : j;
  const float* p = a.cp + c * a.k * 2;
  const float p0x = p[0], p0y = p[1];
  vx = p[2 * pend] - p0x;
  vy = p[2 * pend + 1] - p0y;
  ux = p[2 * mid] - p0x;
  uy = p[2 * mid + 1] - p0y;
  denom = vx * vx + vy * vy + 1e-8f;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + cs_expf(-x)); }

// (side, position) in xyz of closed-path index f (f < M: first half as is;
// else the second half reversed).
__device__ __forceinline__ long long path_offset(const RegArgs& a, long long c, long long f) {
  const long long len = 2 * a.m;
  const long long side = f < a.m ? 0 : 1;
  const long long pos = f < a.m ? f : len - 1 - f;
  return ((c * 2 + side) * a.m + pos) * 2;
}

__device__ __forceinline__ bool curvature_terms(const RegArgs& a, long long t, long long& c,
                                                long long& op_, long long& oc, long long& on,
                                                float& sx, float& sy) {
  c = t / a.per_curve;
  const long long f = (t - c * a.per_curve) * a.stride;
  const long long len = 2 * a.m;
  const long long fp = (f - kRegRoll % len + len) % len, fn = (f + kRegRoll) % len;
  op_ = path_offset(a, c, fp);
  oc = path_offset(a, c, f);
  on = path_offset(a, c, fn);
  const float px = a.xyz[op_], py = a.xyz[op_ + 1];
  const float cx = a.xyz[oc], cy = a.xyz[oc + 1];
  const float nx = a.xyz[on], ny = a.xyz[on + 1];
  sx = px - 2.0f * cx + nx;
  sy = py - 2.0f * cy + ny;
  const float v1x = px - cx, v1y = py - cy, v2x = nx - cx, v2y = ny - cy;
  const float n1 = sqrtf(v1x * v1x + v1y * v1y + 1e-8f);
  const float n2 = sqrtf(v2x * v2x + v2y * v2y + 1e-8f);
  float dot = (v1x / n1) * (v2x / n2) + (v1y / n1) * (v2y / n2);
  dot = fminf(1.0f, fmaxf(-1.0f, dot));
  return dot > a.cos_thresh;
}

__global__ void __launch_bounds__(kRegThreads) reg_forward_kernel(const RegArgs a,
                                                                  float* __restrict__ partial,
                                                                  unsigned* __restrict__ ticket,
                                                                  float* __restrict__ loss) {
  __shared__ float red[kRegThreads / 32];
  __shared__ bool last;
  const long long total = a.t_shape + a.t_op + a.t_bound + a.t_curv;
  float acc = 0.0f;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    long long r = t;
    if (r < a.t_shape) {
      long long c;
      int mid, pend;
      float vx, vy, ux, uy, denom;
      shape_geometry(a, r, c, mid, pend, vx, vy, ux, uy, denom);
      const float al = (ux * vx + uy * vy) / denom;  // the forward's alpha, :46-47
      const float pos = fmaxf(al - 1.0f, 0.0f), neg = fmaxf(-al, 0.0f);
      acc += a.w_shape * (pos * pos + neg * neg);
      continue;
    }
    r -= a.t_shape;
    if (r < a.t_op) {
      acc += a.w_op * fabsf(sigmoidf_(a.op[r]) - 1.0f);
      continue;
    }
    r -= a.t_op;
    if (r < a.t_bound) {
      const long long c = r / (a.joints * 2);
      const long long rem = r - c * a.joints * 2;
      const long long jt = rem >> 1;
      const float x = a.cp[(c * a.k + jt * a.bdeg) * 2 + (rem & 1)];
      acc += a.w_bound * (fmaxf(x - a.bound, 0.0f) + fmaxf(-a.bound - x, 0.0f));
      continue;
    }
    r -= a.t_bound;
    long long c, o0, o1, o2;
    float sx, sy;
    if (curvature_terms(a, r, c, o0, o1, o2, sx, sy)) acc += a.w_curv * (sx * sx + sy * sy);
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int w = 0; w < kRegThreads / 32; ++w) s += red[w];
    partial[blockIdx.x] = s;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    double s = 0.0;
    for (unsigned b = 0; b < gridDim.x; ++b) s += (double)__ldcg(partial + b);
    *loss = (float)s;
    *ticket = 0u;
  }
}

__global__ void __launch_bounds__(kRegThreads) reg_backward_kernel(const RegArgs a,
                                                                   const float* __restrict__ gout,
                                                                   float* __restrict__ g_cp,
                                                                   float* __restrict__ g_op,
                                                                   float* __restrict__ g_xyz) {
  const float go = gout ? *gout : 1.0f;
  const long long total = a.t_shape + a.t_op + a.t_bound + a.t_curv;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    long long r = t;
    if (r < a.t_shape) {
      long long c;
      int mid, pend;
      float vx, vy, ux, uy, denom;
      shape_geometry(a, r, c, mid, pend, vx, vy, ux, uy, denom);
      const float inv_d = 1.0f / denom;
      const float al = (ux * vx + uy * vy) * inv_d;  // the backward's alpha, :70-72
      const float da = al > 1.0f ? 2.0f * (al - 1.0f) : (al < 0.0f ? 2.0f * al : 0.0f);
      const float ds = da * (a.w_shape * go);
      if (ds != 0.0f && g_cp) {
        const float g0 = ds * vx * inv_d, g1 = ds * vy * inv_d;
        const float g2 = ds * (ux * inv_d - 2.0f * al * vx * inv_d);
        const float g3 = ds * (uy * inv_d - 2.0f * al * vy * inv_d);
        float* g = g_cp + c * a.k * 2;
        atomicAdd(g + 0, -(g0 + g2));
        atomicAdd(g + 1, -(g1 + g3));
        atomicAdd(g + 2 * pend, g2);
        atomicAdd(g + 2 * pend + 1, g3);
        atomicAdd(g + 2 * mid, g0);
        atomicAdd(g + 2 * mid + 1, g1);
      }
      continue;
    }
    r -= a.t_shape;
    if (r < a.t_op) {
      if (g_op) {
        const float sig = sigmoidf_(a.op[r]);
        const float d = sig - 1.0f;
        const float sg = d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f);
        g_op[r] = (a.w_op * go) * sg * sig * (1.0f - sig);
      }
      continue;
    }
    r -= a.t_op;
    if (r < a.t_bound) {
      const long long c = r / (a.joints * 2);
      const long long rem = r - c * a.joints * 2;
      const long long idx = (c * a.k + (rem >> 1) * a.bdeg) * 2 + (rem & 1);
      const float x = a.cp[idx];
      const float s = a.w_bound * go;
      const float g = x > a.bound ? s : (x < -a.bound ? -s : 0.0f);
      if (g != 0.0f && g_cp) atomicAdd(g_cp + idx, g);
      continue;
    }
    r -= a.t_bound;
    long long c, o0, o1, o2;
    float sx, sy;
    if (g_xyz && curvature_terms(a, r, c, o0, o1, o2, sx, sy)) {
      const float s = 2.0f * a.w_curv * go;  // d |sec|^2 / d sec = 2 sec
      const float dx = s * sx, dy = s * sy;
      atomicAdd(g_xyz + o0, dx);
      atomicAdd(g_xyz + o0 + 1, dy);
      atomicAdd(g_xyz + o1, -2.0f * dx);
      atomicAdd(g_xyz + o1 + 1, -2.0f * dy);
      atomicAdd(g_xyz + o2, dx);
      atomicAdd(g_xyz + o2 + 1, dy);
    }
  }
}

inline int reg_grid(long long total) {
  const long long b = (total + kRegThreads - 1) / kRegThreads;
  return (int)(b < 1 ? 1 : (b > 148 * 8 ? 148 * 8 : b));
}

// Validates the arguments and fills a; CS_OK or CS_ERR_ARG.
inline int reg_args(RegArgs& a, const float* cp, const float* op, const float* xyz, int64_t n,
                    int64_t k, int64_t n_op, int64_t m, int32_t closed, int32_t split,
                    int32_t bdeg, float bound, int32_t stride, float cos_thresh,
                    float lambda_proj, float opacity_weight) {
  if (n <= 0 || k < 0 || n_op < 0 || !cp || (n_op > 0 && !op)) return CS_ERR_ARG;
  a.cp = cp;
  a.op = op;
  a.xyz = xyz;
  a.n = n;
  a.k = k;
  a.n_op = n_op;
  a.m = closed ? m : 0;
  a.closed = closed ? 1 : 0;
  a.split = split;
  a.bdeg = bdeg;
  a.stride = stride;
  a.bound = bound;
  a.cos_thresh = cos_thresh;
  a.t_shape = k > 2 ? n * (k - 2) : 0;
  if (closed && k > 2 && (split <= 0 || split >= k - 1)) return CS_ERR_ARG;
  a.t_op = n_op;
  a.joints = 0;
  a.per_curve = 0;
  a.t_bound = 0;
  a.t_curv = 0;
  if (closed) {
    if (bdeg <= 0 || stride <= 0 || m < 0 || (m > 0 && !xyz)) return CS_ERR_ARG;
    a.joints = (k + bdeg - 1) / bdeg;
    a.t_bound = n * a.joints * 2;
    a.per_curve = m > 0 ? (2 * m + stride - 1) / stride : 0;
    a.t_curv = n * a.per_curve;
  }
  a.w_shape = lambda_proj / (float)n;
  a.w_op = n_op > 0 ? opacity_weight / (float)n_op : 0.0f;
  a.w_bound = a.joints > 0 ? 1.0f / (float)(n * a.joints * 2) : 0.0f;
  a.w_curv = a.per_curve > 0 ? 1.0f / (float)(n * a.per_curve) : 0.0f;
  return CS_OK;
}

}  // namespace cs

using namespace cs;

extern "C" {

size_t cs_regularization_workspace_size(void) {
  return sizeof(float) * 148 * 8 + 256;
}

int cs_regularization_forward(const float* control_points, const float* opacity,
                              const float* xyz, int64_t num_curves, int64_t num_ctrl,
                              int64_t num_opacity, int64_t points_per_side, int32_t closed,
                              int32_t split_idx, int32_t boundary_degree, float boundary_bound,
                              int32_t curvature_stride, float curvature_cos_thresh,
                              float lambda_proj, float opacity_weight, float* loss,
                              void* workspace, void* stream) {
  RegArgs a;
  if (!loss || !workspace) return CS_ERR_ARG;
  const int rc = reg_args(a, control_points, opacity, xyz, num_curves, num_ctrl, num_opacity,
                          points_per_side, closed, split_idx, boundary_degree, boundary_bound,
                          curvature_stride, curvature_cos_thresh, lambda_proj, opacity_weight);
  if (rc != CS_OK) return rc;
  const long long total = a.t_shape + a.t_op + a.t_bound + a.t_curv;
  float* partial = static_cast<float*>(workspace);
  unsigned* ticket = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) +
                                                 sizeof(float) * 148 * 8);
  reg_forward_kernel<<<reg_grid(total), kRegThreads, 0, (cudaStream_t)stream>>>(a, partial,
                                                                                ticket, loss);
  return launch_status();
}

int cs_regularization_backward(const float* control_points, const float* opacity,
                               const float* xyz, int64_t num_curves, int64_t num_ctrl,
                               int64_t num_opacity, int64_t points_per_side, int32_t closed,
                               int32_t split_idx, int32_t boundary_degree, float boundary_bound,
                               int32_t curvature_stride, float curvature_cos_thresh,
                               float lambda_proj, float opacity_weight, const float* grad_output,
                               float* grad_control_points, float* grad_opacity, float* grad_xyz,
                               void* stream) {
  RegArgs a;
  const int rc = reg_args(a, control_points, opacity, xyz, num_curves, num_ctrl, num_opacity,
                          points_per_side, closed, split_idx, boundary_degree, boundary_bound,
                          curvature_stride, curvature_cos_thresh, lambda_proj, opacity_weight);
  if (rc != CS_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (grad_control_points)
    cudaMemsetAsync(grad_control_points, 0, sizeof(float) * num_curves * num_ctrl * 2, st);
  if (grad_xyz && a.closed && a.m > 0)
    cudaMemsetAsync(grad_xyz, 0, sizeof(float) * num_curves * 4 * a.m, st);
  const long long total = a.t_shape + a.t_op + a.t_bound + a.t_curv;
  reg_backward_kernel<<<reg_grid(total), kRegThreads, 0, st>>>(
      a, grad_output, grad_control_points, grad_opacity, a.closed ? grad_xyz : nullptr);
  return launch_status();
}

}  // extern "C"
