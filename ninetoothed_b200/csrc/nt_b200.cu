// libnt_b200.so: B200 (sm_100a) kernels for the operator programs NineToothed's
// arrange-and-apply API generates.  The library is one translation unit so the
// device error word is shared by every kernel without relocatable device code.
#include <cuda_runtime.h>

#include "common.cuh"
#include "softmax.cuh"
#include "elementwise.cuh"
#include "pool.cuh"
#include "copy.cuh"
#include "contractions.cuh"
#include "conv_no_alloc.cu"

namespace nt {

int sm_count() {
  static std::atomic<int> cached[64] = {};  // per device, filled on first use (any thread)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

namespace tc {
EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}
EncodeIm2colFn encode_im2col_fn() {
  static EncodeIm2colFn fn = []() -> EncodeIm2colFn {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeIm2colFn>(ptr);
  }();
  return fn;
}
}  // namespace tc

}  // namespace nt

extern "C" int nt_b200_version(void) { return 1; }

extern "C" const char *nt_b200_error_string(int code) {
  switch (code) {
    case 0: return "success";
    case NT_B200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NT_B200_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case NT_B200_ERR_SHAPE_MISMATCH: return "shape mismatch";
    case NT_B200_ERR_NO_DEVICE: return "no sm_100 device";
    case NT_B200_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
    case NT_B200_ERR_WORKSPACE_TOO_LARGE: return "conv2d staging exceeds the library's fixed 64 MiB array";
    default: return cudaGetErrorString(static_cast<cudaError_t>(code));
  }
}

extern "C" int nt_b200_device_status(void *stream, int *status) {
  if (!status) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  const int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&host, nt::g_error_word, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(nt::g_error_word, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return static_cast<int>(e);
  *status = host;
  return 0;
}

// Self-test of the bounded waits: one thread waits on an mbarrier that nothing
// ever arrives on, with a short limit, so the wait runs out the same way a
// broken pipeline's would.
namespace nt {
__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&bar), 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) ptx::mbar_wait(ptx::smem_u32(&bar), 0, &abort_flag, limit_ns);
}
}  // namespace nt

extern "C" int nt_b200_wait_timeout_selftest(int64_t limit_ns, void *stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000LL) return NT_B200_ERR_INVALID_ARGUMENT;
  nt::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>((uint64_t)limit_ns);
  return nt::launch_status();
}
