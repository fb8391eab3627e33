// nt_b200_conv2d_no_alloc: conv2d for callers that cannot hand the library a
// workspace.
//
// nt_b200_conv2d stages the input (W-padded NHWC) and the filter (KRSC) in device memory
// the caller passes in.  Some callers have no way to provide it at call time: a
// plain C host program that owns no device allocator, a serving loop that must
// not call cudaMalloc because it synchronises the whole device and stalls every
// other stream, or an application that reserves its whole memory budget once at
// start-up.  This entry point takes the staging memory from a fixed array that
// lives inside the library instead, so a call allocates nothing.
//
// Limits and sharing:
//   - the array holds kConvStaticWorkspaceBytes (64 MiB) on every GPU that loads
//     the library, for as long as the process runs;
//   - problems whose staging needs more are rejected with
//     NT_B200_ERR_WORKSPACE_TOO_LARGE before anything is launched;
//   - all calls on a device share the one array: two calls whose kernels
//     overlap on the GPU (different streams, no ordering between them) race on
//     it and corrupt each other's results.  Calls on one stream are ordered and
//     safe.  The staging writes every byte it later reads, so the contents left
//     by the previous call never leak into a result;
//   - the device address of the array is looked up (cudaGetSymbolAddress) the
//     first time the entry point runs on a device, with that device current,
//     and again on later calls until a lookup succeeds; make that first call
//     before any stream capture begins, and do not use the entry point on a
//     device after cudaDeviceReset in the same process.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace nt {
namespace no_alloc {

constexpr int64_t kConvStaticWorkspaceBytes = int64_t(64) << 20;
constexpr int kMaxDevices = 64;

// Staging memory of nt_b200_conv2d_no_alloc (one instance per device).  Host
// code may not pass `g_conv_scratch` itself to a kernel: on the host that name
// is only a stand-in, not a device address; use scratch_address().
static __device__ __align__(256) uint8_t g_conv_scratch[kConvStaticWorkspaceBytes];

// The address is published through an atomic once a lookup has succeeded; a
// failed lookup (say, a first call made while the device's context could not
// be created) is not remembered, so a later call on that device tries again.
struct DeviceScratch {
  std::mutex lock;
  std::atomic<void *> address{nullptr};
};

static DeviceScratch g_device_scratch[kMaxDevices];

// Device address of g_conv_scratch on the current device, looked up with that
// device current until one lookup succeeds.  Returns 0 or an error code.
static int scratch_address(void **out) {
  int device = 0;
  const cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (device < 0 || device >= kMaxDevices) return NT_B200_ERR_NO_DEVICE;
  DeviceScratch &slot = g_device_scratch[device];
  void *address = slot.address.load(std::memory_order_acquire);
  if (address == nullptr) {
    std::lock_guard<std::mutex> guard(slot.lock);
    address = slot.address.load(std::memory_order_acquire);
    if (address == nullptr) {
      const cudaError_t status = cudaGetSymbolAddress(&address, g_conv_scratch);
      if (status != cudaSuccess || address == nullptr) {
        cudaGetLastError();  // the failed lookup leaves no sticky error behind for the caller's next launch
        return static_cast<int>(status != cudaSuccess ? status : cudaErrorInvalidSymbol);
      }
      slot.address.store(address, std::memory_order_release);
    }
  }
  *out = address;
  return 0;
}

}  // namespace no_alloc
}  // namespace nt

extern "C" int nt_b200_conv2d_no_alloc(const void *input, const void *filter, void *output, int64_t n, int64_t c,
                                       int64_t h, int64_t w, int64_t k, int64_t r, int64_t s, int64_t pad_h,
                                       int64_t pad_w, const int64_t *input_strides, const int64_t *filter_strides,
                                       const int64_t *output_strides, int dtype, void *stream) {
  const int64_t need = nt_b200_conv2d_workspace_size(n, c, h, w, k, r, s, pad_h, pad_w, dtype);
  if (need > nt::no_alloc::kConvStaticWorkspaceBytes) return NT_B200_ERR_WORKSPACE_TOO_LARGE;
  void *scratch = nullptr;
  if (need > 0 && n * k * (h + 2 * pad_h - r + 1) * (w + 2 * pad_w - s + 1) > 0) {
    const int rc = nt::no_alloc::scratch_address(&scratch);
    if (rc != 0) return rc;
  }
  return nt_b200_conv2d(input, filter, output, n, c, h, w, k, r, s, pad_h, pad_w, input_strides, filter_strides,
                        output_strides, scratch, scratch ? need : 0, dtype, stream);
}
