// Cross-GPU exchange over peer memory (NVLink / NVSwitch) for one image split
// across ranks in tile-row bands, one process per GPU.
//
// Every rank owns a symmetric buffer (the same layout on every rank, each
// rank holding device pointers to all the others'): flag words, this rank's
// gradients of the step (double-buffered by step parity) and the first rows
// of its band for the next band's SSIM window.  Instead of a library
// all-reduce followed by a replicated optimiser step, one kernel waits for
// every rank's "gradients ready" flag, reads all ranks' gradients through
// peer pointers, sums them in rank order (so every rank gets bit-identical
// sums and identical parameters), applies Adam and clears this rank's buffer
// of the next parity.  A flag is a step number stored with release
// semantics at system scope after the data it guards; readers poll their own
// flag words with acquire loads.  Every wait is bounded: on timeout it
// records CS_ERR_TIMEOUT in the caller's status word and the kernel skips its
// work instead of hanging.  Nothing here is a TMA or bulk copy: peer data is
// read with plain loads that bypass L1.
#include <algorithm>

#include "cs_common.cuh"

namespace cs {

__device__ __forceinline__ void st_release_sys(unsigned* addr, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Whether flag word `slot * world + q` of this rank has reached `target`
// for every rank q (or only for rank `only` when only >= 0), polling at most
// `limit` times.  Flags count steps, so the comparison is a signed difference.
__device__ bool wait_flags(const unsigned* flags, int slot, int world, unsigned target, int only,
                           long long limit) {
  for (long long it = 0; it < limit; ++it) {
    bool ok = true;
    for (int q = 0; q < world; ++q) {
      if (only >= 0 && q != only) continue;
      const unsigned v = ld_acquire_sys(flags + slot * world + q);
      ok &= (int)(v - target) >= 0;
    }
    if (ok) return true;
    __nanosleep(64);
  }
  return false;
}

__global__ void peer_signal_kernel(const unsigned long long* __restrict__ flag_ptrs, int rank,
                                   int world, int slot, const int* __restrict__ epoch, int add,
                                   int only) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const unsigned v = (unsigned)(*epoch + add);
  __threadfence_system();  // the stream's earlier writes first, then the flags
  for (int q = 0; q < world; ++q) {
    if (only >= 0 && q != only) continue;
    unsigned* f = reinterpret_cast<unsigned*>(flag_ptrs[q]) + slot * world + rank;
    st_release_sys(f, v);
  }
}

// Waits for rank `from`'s flag, then copies `planes` blocks of `plane_elems`
// floats from src (strided by src_stride) to dst (strided by dst_stride).
__global__ void peer_wait_copy_kernel(const unsigned* __restrict__ flags, int slot, int world,
                                      int from, const int* __restrict__ epoch, int add,
                                      long long limit, int* __restrict__ status,
                                      const float* __restrict__ src, long long src_stride,
                                      float* __restrict__ dst, long long dst_stride,
                                      long long plane_elems, int planes) {
  __shared__ bool ok;
  if (threadIdx.x == 0) {
    ok = wait_flags(flags, slot, world, (unsigned)(*epoch + add), from, limit);
    if (!ok && status) atomicExch(status, CS_ERR_TIMEOUT);
  }
  __syncthreads();
  if (!ok || src == nullptr) return;
  const long long total = plane_elems * planes;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long pl = i / plane_elems, e = i - pl * plane_elems;
    dst[pl * dst_stride + e] = __ldcg(src + pl * src_stride + e);
  }
}

// Sum over ranks (in rank order) of element i of every rank's gradients.
__device__ __forceinline__ float rank_sum(const unsigned long long* __restrict__ grad_ptrs,
                                          int world, long long i) {
  float g = 0.0f;
  for (int q = 0; q < world; ++q) g = g + __ldcg(reinterpret_cast<const float*>(grad_ptrs[q]) + i);
  return g;
}

__device__ __forceinline__ float4 rank_sum4(const unsigned long long* __restrict__ grad_ptrs,
                                            int world, long long i4) {
  float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q = 0; q < world; ++q) {
    const float4 x = __ldcg(reinterpret_cast<const float4*>(grad_ptrs[q]) + i4);
    g.x = g.x + x.x;
    g.y = g.y + x.y;
    g.z = g.z + x.z;
    g.w = g.w + x.w;
  }
  return g;
}

__global__ void __launch_bounds__(256) allreduce_adam_kernel(
    const unsigned long long* __restrict__ grad_ptrs, int world, float* __restrict__ p,
    float* __restrict__ m, float* __restrict__ v, long long n, long long n_first, int n_tail,
    float* __restrict__ tail_out, float* __restrict__ clear_buf, float lr0, float lr1, float b1,
    float b2, float eps, int* __restrict__ step, const unsigned* __restrict__ flags, int slot,
    long long limit, int* __restrict__ status, unsigned* __restrict__ ticket, int vec4) {
  __shared__ bool ok, last;
  const int t = *step + 1;
  if (threadIdx.x == 0) {
    ok = wait_flags(flags, slot, world, (unsigned)t, -1, limit);
    if (!ok && status) atomicExch(status, CS_ERR_TIMEOUT);
  }
  __syncthreads();
  if (ok) {
    const float bc1 = 1.0f - powf(b1, (float)t);
    const float bc2 = 1.0f - powf(b2, (float)t);
    const float rb2 = 1.0f / sqrtf(bc2);
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec4) {  // n and every buffer 16-byte aligned: four elements per thread
      for (long long i4 = tid; i4 < n / 4; i4 += stride) {
        const float4 g = rank_sum4(grad_ptrs, world, i4);
        float4 pp = reinterpret_cast<float4*>(p)[i4];
        float4 mm = reinterpret_cast<float4*>(m)[i4];
        float4 vv = reinterpret_cast<float4*>(v)[i4];
        const long long i = 4 * i4;
        adam_element(pp.x, mm.x, vv.x, g.x, i < n_first ? lr0 : lr1, b1, b2, eps, bc1, rb2);
        adam_element(pp.y, mm.y, vv.y, g.y, i + 1 < n_first ? lr0 : lr1, b1, b2, eps, bc1, rb2);
        adam_element(pp.z, mm.z, vv.z, g.z, i + 2 < n_first ? lr0 : lr1, b1, b2, eps, bc1, rb2);
        adam_element(pp.w, mm.w, vv.w, g.w, i + 3 < n_first ? lr0 : lr1, b1, b2, eps, bc1, rb2);
        reinterpret_cast<float4*>(p)[i4] = pp;
        reinterpret_cast<float4*>(m)[i4] = mm;
        reinterpret_cast<float4*>(v)[i4] = vv;
        if (clear_buf) reinterpret_cast<float4*>(clear_buf)[i4] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    } else {
      for (long long i = tid; i < n; i += stride) {
        const float g = rank_sum(grad_ptrs, world, i);
        adam_element(p[i], m[i], v[i], g, i < n_first ? lr0 : lr1, b1, b2, eps, bc1, rb2);
        if (clear_buf) clear_buf[i] = 0.0f;
      }
    }
    if (blockIdx.x == 0 && threadIdx.x < n_tail) {  // loss and metric sums after the gradients
      const long long i = n + threadIdx.x;
      if (tail_out) tail_out[threadIdx.x] = rank_sum(grad_ptrs, world, i);
      if (clear_buf) clear_buf[i] = 0.0f;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    if (ok) *step = t;
    *ticket = 0u;
  }
}

inline bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace cs

using namespace cs;

extern "C" {

size_t cs_allreduce_adam_workspace_size(void) { return 256; }

int cs_peer_signal(const uint64_t* flag_ptrs, int32_t rank, int32_t world, int32_t slot,
                   const int32_t* epoch, int32_t epoch_add, int32_t only_peer, void* stream) {
  if (!flag_ptrs || !epoch || world <= 0 || rank < 0 || rank >= world || slot < 0 ||
      only_peer >= world)
    return CS_ERR_ARG;
  peer_signal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const unsigned long long*>(flag_ptrs), rank, world, slot, epoch, epoch_add,
      only_peer);
  return launch_status();
}

int cs_peer_wait_copy(const uint32_t* flags, int32_t slot, int32_t world, int32_t from_rank,
                      const int32_t* epoch, int32_t epoch_add, int64_t spin_limit,
                      int32_t* status, const float* src, int64_t src_plane_stride, float* dst,
                      int64_t dst_plane_stride, int64_t plane_elems, int32_t planes,
                      void* stream) {
  if (!flags || !epoch || world <= 0 || from_rank < 0 || from_rank >= world || slot < 0 ||
      spin_limit <= 0 || plane_elems < 0 || planes < 0 || (src && !dst))
    return CS_ERR_ARG;
  const long long total = plane_elems * planes;
  const int blocks = (int)std::min<long long>(std::max<long long>(1, (total + 255) / 256), 148);
  peer_wait_copy_kernel<<<src ? blocks : 1, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const unsigned*>(flags), slot, world, from_rank, epoch, epoch_add,
      spin_limit, status, src, src_plane_stride, dst, dst_plane_stride, plane_elems, planes);
  return launch_status();
}

int cs_allreduce_adam(const uint64_t* grad_ptrs, int32_t world, float* params, float* exp_avg,
                      float* exp_avg_sq, int64_t n, int64_t n_first, int32_t n_tail,
                      float* tail_out, float* clear_buf, float lr_first, float lr_rest,
                      float beta1, float beta2, float eps, int32_t* step, const uint32_t* flags,
                      int32_t flag_slot, int64_t spin_limit, int32_t* status, void* workspace,
                      void* stream) {
  if (!grad_ptrs || world <= 0 || !params || !exp_avg || !exp_avg_sq || n < 0 || n_first < 0 ||
      n_tail < 0 || n_tail > 256 || !step || !flags || flag_slot < 0 || spin_limit <= 0 ||
      !workspace)
    return CS_ERR_ARG;
  const bool vec4 = (n % 4 == 0) && al16(params) && al16(exp_avg) && al16(exp_avg_sq) &&
                    (!clear_buf || al16(clear_buf));
  const long long work = vec4 ? n / 4 : n;
  const int blocks = (int)std::min<long long>(std::max<long long>(1, (work + 255) / 256), 148 * 4);
  allreduce_adam_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const unsigned long long*>(grad_ptrs), world, params, exp_avg,
      exp_avg_sq, n, n_first, n_tail, tail_out, clear_buf, lr_first, lr_rest, beta1, beta2, eps,
      step, reinterpret_cast<const unsigned*>(flags), flag_slot, spin_limit, status,
      static_cast<unsigned*>(workspace), vec4 ? 1 : 0);
  return launch_status();
}

}  // extern "C"
