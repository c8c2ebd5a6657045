// 4-connected component labelling of a uint8 mask (sm_100a), behind
// connected_components_labels_4_tilelang / _with_stats_4_tilelang
// (manbo/ops/connected_components.py:98-236).
//
// The reference relaxes every label to the minimum of its 4-neighbours, one
// launch and one host read per sweep, until nothing changes (up to 4096
// sweeps); a component ends labelled with its smallest linear index + 1.
// Here a union-find gives the same labels in three launches: every
// foreground pixel starts as its own root, every foreground pixel joins its
// left and upper foreground neighbours (roots are linked with atomicMin, so a
// root only ever points to a smaller index and the smallest index of a
// component stays its root), and a final pass points every pixel at its
// root.  Each union retries a bounded number of times; past the bound the
// status word is set (it cannot happen for parents that only decrease, but
// no loop here is unbounded).
//
// The statistics pass accumulates, per root, the area, coordinate sums and
// bounding box with atomics; a scan over the roots in raster order numbers
// the components 1.. as the reference's renumbering does, and a gather writes
// stats [x, y, width, height, area] and float32 centres [mean x, mean y].

#include "cs_common.cuh"

namespace cs {

constexpr int kCclThreads = 256;
constexpr int kCclScanItems = 4;                       // per thread
constexpr int kCclScanBlock = kCclThreads * kCclScanItems;
constexpr int kCclMaxSteps = 1 << 22;

struct CclWs {
  int* parent;
  int* area;
  int* minx;
  int* miny;
  int* maxx;
  int* maxy;
  int* id;
  unsigned long long* sx;
  unsigned long long* sy;
  int* bsum;  // [blocks + 1]
};

__host__ __device__ inline size_t ccl_al(size_t v) { return (v + 255) & ~size_t(255); }

inline long long ccl_blocks(long long n) { return (n + kCclScanBlock - 1) / kCclScanBlock; }

inline size_t ccl_ws_size(long long n) {
  const size_t i = ccl_al(sizeof(int) * (size_t)n), u = ccl_al(sizeof(unsigned long long) * n);
  return 7 * i + 2 * u + ccl_al(sizeof(int) * (size_t)(ccl_blocks(n) + 1));
}

inline CclWs ccl_ws(void* base, long long n) {
  char* b = static_cast<char*>(base);
  const size_t i = ccl_al(sizeof(int) * (size_t)n), u = ccl_al(sizeof(unsigned long long) * n);
  CclWs w;
  w.parent = reinterpret_cast<int*>(b);
  w.area = reinterpret_cast<int*>(b + i);
  w.minx = reinterpret_cast<int*>(b + 2 * i);
  w.miny = reinterpret_cast<int*>(b + 3 * i);
  w.maxx = reinterpret_cast<int*>(b + 4 * i);
  w.maxy = reinterpret_cast<int*>(b + 5 * i);
  w.id = reinterpret_cast<int*>(b + 6 * i);
  w.sx = reinterpret_cast<unsigned long long*>(b + 7 * i);
  w.sy = reinterpret_cast<unsigned long long*>(b + 7 * i + u);
  w.bsum = reinterpret_cast<int*>(b + 7 * i + 2 * u);
  return w;
}

// Root of x (parents only decrease along a chain); -1 past the step bound.
__device__ __forceinline__ int ccl_find(const int* parent, int x) {
  for (int s = 0; s < kCclMaxSteps; ++s) {
    const int p = __ldcg(parent + x);
    if (p == x) return x;
    x = p;
  }
  return -1;
}

__device__ __forceinline__ void ccl_unite(int* parent, int a, int b, int* status) {
  for (int s = 0; s < kCclMaxSteps; ++s) {
    a = ccl_find(parent, a);
    b = ccl_find(parent, b);
    if (a < 0 || b < 0) break;
    if (a == b) return;
    if (a < b) {
      const int t = a;
      a = b;
      b = t;
    }
    const int old = atomicMin(parent + a, b);  // link the larger root under the smaller
    if (old == a) return;
    a = old;
  }
  atomicExch(status, CS_ERR_CUDA);
}

__global__ void ccl_init_kernel(const uint8_t* __restrict__ mask, int* __restrict__ parent,
                                long long n) {
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p < n) parent[p] = mask[p] ? (int)p : -1;
}

__global__ void ccl_merge_kernel(const uint8_t* __restrict__ mask, int* parent, int h, int w,
                                 int* status) {
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= (long long)h * w || !mask[p]) return;
  const int x = (int)(p % w), y = (int)(p / w);
  if (x > 0 && mask[p - 1]) ccl_unite(parent, (int)p, (int)p - 1, status);
  if (y > 0 && mask[p - w]) ccl_unite(parent, (int)p, (int)(p - w), status);
}

__global__ void ccl_flatten_kernel(const uint8_t* __restrict__ mask, int* parent,
                                   int* __restrict__ labels, long long n, int* status) {
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  if (!mask[p]) {
    labels[p] = 0;
    return;
  }
  const int r = ccl_find(parent, (int)p);
  if (r < 0) {
    atomicExch(status, CS_ERR_CUDA);
    labels[p] = 0;
    return;
  }
  labels[p] = r + 1;
}

__global__ void ccl_stats_init_kernel(CclWs ws, long long n, int h, int w) {
  const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  ws.area[r] = 0;
  ws.minx[r] = w;
  ws.miny[r] = h;
  ws.maxx[r] = -1;
  ws.maxy[r] = -1;
  ws.sx[r] = 0ull;
  ws.sy[r] = 0ull;
}

// Per-root accumulation from raw labels (root + 1; 0 = background).  Labels
// outside [0, n] are ignored (status set).
__global__ void ccl_stats_acc_kernel(const int* __restrict__ labels, CclWs ws, int h, int w,
                                     int* status) {
  const long long n = (long long)h * w;
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const int l = labels[p];
  if (l == 0) return;
  if (l < 0 || (long long)l > n) {
    atomicExch(status, CS_ERR_ARG);
    return;
  }
  const int r = l - 1;
  const int x = (int)(p % w), y = (int)(p / w);
  atomicAdd(ws.area + r, 1);
  atomicAdd(ws.sx + r, (unsigned long long)x);
  atomicAdd(ws.sy + r, (unsigned long long)y);
  atomicMin(ws.minx + r, x);
  atomicMin(ws.miny + r, y);
  atomicMax(ws.maxx + r, x);
  atomicMax(ws.maxy + r, y);
}

// Block-local exclusive scan of the root flags (area > 0) into id, block
// totals into bsum.
__global__ void __launch_bounds__(kCclThreads) ccl_scan_local_kernel(CclWs ws, long long n) {
  __shared__ int wsum[kCclThreads / 32];
  const long long b0 = (long long)blockIdx.x * kCclScanBlock + (long long)threadIdx.x * kCclScanItems;
  int f[kCclScanItems], local = 0;
#pragma unroll
  for (int q = 0; q < kCclScanItems; ++q) {
    f[q] = b0 + q < n && ws.area[b0 + q] > 0 ? 1 : 0;
    local += f[q];
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int incl = warp_incl_scan(local, lane);
  if (lane == 31) wsum[wid] = incl;
  __syncthreads();
  int base = 0, total = 0;
#pragma unroll
  for (int k = 0; k < kCclThreads / 32; ++k) {
    base += k < wid ? wsum[k] : 0;
    total += wsum[k];
  }
  int run = base + incl - local;
#pragma unroll
  for (int q = 0; q < kCclScanItems; ++q) {
    if (b0 + q < n) ws.id[b0 + q] = run;
    run += f[q];
  }
  if (threadIdx.x == 0) ws.bsum[blockIdx.x] = total;
}

// One CTA: exclusive scan of the block totals in place; the component count
// into *count.
__global__ void __launch_bounds__(1024) ccl_scan_blocks_kernel(CclWs ws, long long nb,
                                                               int* __restrict__ count) {
  __shared__ int wsum[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (long long c0 = 0; c0 < nb; c0 += 1024) {
    const long long i = c0 + threadIdx.x;
    const int v = i < nb ? ws.bsum[i] : 0;
    const int incl = warp_incl_scan(v, lane);
    if (lane == 31) wsum[wid] = incl;
    __syncthreads();
    int base = 0, total = 0;
    for (int k = 0; k < 32; ++k) {
      base += k < wid ? wsum[k] : 0;
      total += wsum[k];
    }
    if (i < nb) ws.bsum[i] = carry + base + incl - v;
    __syncthreads();
    if (threadIdx.x == 0) carry += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = carry;
}

__global__ void ccl_compact_kernel(const int* __restrict__ labels, CclWs ws,
                                   int* __restrict__ out, long long n) {
  const long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const int l = labels[p];
  if (l <= 0 || (long long)l > n) {
    out[p] = 0;
    return;
  }
  const long long r = l - 1;
  out[p] = ws.bsum[r / kCclScanBlock] + ws.id[r] + 1;
}

__global__ void ccl_gather_kernel(CclWs ws, long long n, int ncomp, int* __restrict__ stats,
                                  float* __restrict__ centres) {
  const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const int a = ws.area[r];
  if (a <= 0) return;
  const int k = ws.bsum[r / kCclScanBlock] + ws.id[r];
  if (k >= ncomp) return;
  const int x0 = ws.minx[r], y0 = ws.miny[r];
  int* s = stats + (long long)k * 5;
  s[0] = x0;
  s[1] = y0;
  s[2] = ws.maxx[r] - x0 + 1;
  s[3] = ws.maxy[r] - y0 + 1;
  s[4] = a;
  centres[2 * (long long)k] = (float)ws.sx[r] / (float)a;
  centres[2 * (long long)k + 1] = (float)ws.sy[r] / (float)a;
}

}  // namespace cs

using namespace cs;

extern "C" {

size_t cs_ccl_workspace_size(int64_t num_pixels) {
  return num_pixels > 0 ? ccl_ws_size(num_pixels) : 256;
}

int cs_ccl_labels_4(const uint8_t* mask, int32_t height, int32_t width, int32_t* labels,
                    int32_t* status, void* workspace, void* stream) {
  if (height < 0 || width < 0 || !status || !workspace) return CS_ERR_ARG;
  const long long n = (long long)height * width;
  if (n == 0) return CS_OK;
  if (!mask || !labels || n >= (1LL << 31) - 1) return CS_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  CclWs ws = ccl_ws(workspace, n);
  const int g = ceil_div(n, kCclThreads);
  ccl_init_kernel<<<g, kCclThreads, 0, st>>>(mask, ws.parent, n);
  ccl_merge_kernel<<<g, kCclThreads, 0, st>>>(mask, ws.parent, height, width, status);
  ccl_flatten_kernel<<<g, kCclThreads, 0, st>>>(mask, ws.parent, labels, n, status);
  return launch_status();
}

int cs_ccl_compact_4(const int32_t* labels, int32_t height, int32_t width,
                     int32_t* labels_compact, int32_t* num_components, int32_t* status,
                     void* workspace, void* stream) {
  if (height < 0 || width < 0 || !num_components || !status || !workspace) return CS_ERR_ARG;
  const long long n = (long long)height * width;
  cudaStream_t st = (cudaStream_t)stream;
  if (n == 0) return cudaMemsetAsync(num_components, 0, sizeof(int32_t), st) == cudaSuccess
                         ? CS_OK : CS_ERR_CUDA;
  if (!labels || !labels_compact || n >= (1LL << 31) - 1) return CS_ERR_ARG;
  CclWs ws = ccl_ws(workspace, n);
  const int g = ceil_div(n, kCclThreads);
  const long long nb = ccl_blocks(n);
  ccl_stats_init_kernel<<<g, kCclThreads, 0, st>>>(ws, n, height, width);
  ccl_stats_acc_kernel<<<g, kCclThreads, 0, st>>>(labels, ws, height, width, status);
  ccl_scan_local_kernel<<<(int)nb, kCclThreads, 0, st>>>(ws, n);
  ccl_scan_blocks_kernel<<<1, 1024, 0, st>>>(ws, nb, num_components);
  ccl_compact_kernel<<<g, kCclThreads, 0, st>>>(labels, ws, labels_compact, n);
  return launch_status();
}

int cs_ccl_stats_4(int32_t height, int32_t width, int32_t num_components, int32_t* stats,
                   float* centers, void* workspace, void* stream) {
  if (height < 0 || width < 0 || num_components < 0 || !workspace) return CS_ERR_ARG;
  const long long n = (long long)height * width;
  if (n == 0 || num_components == 0) return CS_OK;
  if (!stats || !centers) return CS_ERR_ARG;
  CclWs ws = ccl_ws(workspace, n);
  ccl_gather_kernel<<<ceil_div(n, kCclThreads), kCclThreads, 0, (cudaStream_t)stream>>>(
      ws, n, num_components, stats, centers);
  return launch_status();
}

}  // extern "C"
