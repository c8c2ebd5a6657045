// Host-runtime helpers of the C ABI for callers that capture the renderer in
// a CUDA graph: a stream-capture query and the guard that makes a captured
// frame whose binning overflowed fail loudly (a NaN image) instead of quietly
// showing the background.
#include "cs_common.cuh"

namespace cs {

// Every element of data becomes NaN when *status is not CS_OK.
__global__ void __launch_bounds__(256) poison_kernel(const int32_t* __restrict__ status,
                                                     float* __restrict__ data, long long n) {
  if (*status == CS_OK) return;
  const float nan = __int_as_float(0x7fc00000);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    data[i] = nan;
}

}  // namespace cs

extern "C" {

int cs_stream_is_capturing(void* stream) {
  cudaStreamCaptureStatus s = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing((cudaStream_t)stream, &s) != cudaSuccess) return -1;
  return s == cudaStreamCaptureStatusNone ? 0 : 1;
}

int cs_poison_on_status(const int32_t* status, float* data, int64_t n, void* stream) {
  if (!status || (n > 0 && !data) || n < 0) return CS_ERR_ARG;
  if (n == 0) return CS_OK;
  const long long blocks = (n + 255) / 256;
  cs::poison_kernel<<<(unsigned)(blocks < 1184 ? blocks : 1184), 256, 0, (cudaStream_t)stream>>>(
      status, data, n);
  return cudaGetLastError() == cudaSuccess ? CS_OK : CS_ERR_CUDA;
}

}  // extern "C"
