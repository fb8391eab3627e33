// Shared helpers for the sm_100a kernels of libnt_b200.so: element conversion,
// argument checks, the device error word and the launch-error convention.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include <atomic>

#include "../../include/nt_b200.h"

namespace nt {

// Opts kernel `Kern` in to `bytes` of dynamic shared memory once per device:
// the first launch on a device sets the attribute, later launches read one
// atomic word.  No lock on the launch path; two host threads that race on a
// device's first launch both set the (idempotent) attribute.
template <auto Kern>
inline cudaError_t smem_optin(int bytes) {
  static std::atomic<uint64_t> done{0};  // bit d: device d has the attribute
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
  e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// Device error word of this library (one per device, zero-initialised at load).
// The library is a single translation unit, so this is its only definition.
__device__ int g_error_word = 0;

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_error_word, 0, code); }

template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr bool is_f16 = false;
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__half> {
  static constexpr bool is_f16 = true;
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr bool is_f16 = false;
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <> struct Elem<__nv_fp8_e4m3> {
  static constexpr bool is_f16 = false;
  static __device__ __forceinline__ float to_f(__nv_fp8_e4m3 v) { return static_cast<float>(v); }
  static __device__ __forceinline__ __nv_fp8_e4m3 from_f(float v) { return __nv_fp8_e4m3(v); }
};
template <> struct Elem<__nv_fp8_e5m2> {
  static constexpr bool is_f16 = false;
  static __device__ __forceinline__ float to_f(__nv_fp8_e5m2 v) { return static_cast<float>(v); }
  static __device__ __forceinline__ __nv_fp8_e5m2 from_f(float v) { return __nv_fp8_e5m2(v); }
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return Elem<T>::to_f(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return Elem<T>::from_f(v); }

// Rounds an fp32 value through float16 (the `.to(ntl.float16)` of the matmul
// application) and returns it as fp32.
__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// The addmm application's epilogue, `beta * input + alpha * matmul_output`, with
// Triton's typing of a scalar kernel argument against a tensor (the tensor's
// dtype wins): beta * input is computed in the input dtype TI, alpha * the
// float16-rounded accumulator in float16, and the sum in float16 when TI is
// float16 (float32 for bfloat16 with float16).  8-bit inputs are the exception:
// beta * input is kept at float16 precision, the only reading under which the
// reference's own float8_e5m2 addmm test (atol 0.125 against a float16
// torch.addmm) can pass -- e5m2 rounding of the product alone errs by up to
// 0.25 there -- and the sum is float16.  `beta_t` and `alpha_h` are the scalars
// already rounded to ScaleType<TI> and float16.  Each fp32 operation here is
// exact or followed by one rounding to a type with at most half fp32's
// precision, so the result is the correctly rounded value of each typed
// operation.
template <typename TI> struct ScaleType { using type = TI; };
template <> struct ScaleType<__nv_fp8_e4m3> { using type = __half; };
template <> struct ScaleType<__nv_fp8_e5m2> { using type = __half; };

template <typename TI>
__device__ __forceinline__ float addmm_value(float beta_t, float alpha_h, float in, float acc) {
  using S = typename ScaleType<TI>::type;
  const float scaled_in = to_f(from_f<S>(beta_t * in));
  const float scaled_mm = round_f16(alpha_h * round_f16(acc));
  if constexpr (sizeof(S) == 2 && Elem<S>::is_f16) return round_f16(scaled_in + scaled_mm);
  return scaled_in + scaled_mm;
}

inline int launch_status() {
  cudaError_t err = cudaGetLastError();
  return static_cast<int>(err);
}

// Programmatic dependent launch.  A kernel launched with launch_overlapped may
// be scheduled while the kernel before it in the stream still runs its last
// CTAs (from the point where every CTA of that kernel has called
// allow_dependent_launch, or at its end), which hides the launch latency of
// short back-to-back kernels.  Such a kernel must call wait_prior_grid before
// it touches global memory: that returns once the previous kernel has
// completed and its writes are visible, so stream order is kept for any
// predecessor.  Kernels that follow without the attribute wait as usual.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline int launch_overlapped(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

inline bool is_float_dtype(int dtype) {
  return dtype == NT_B200_FLOAT16 || dtype == NT_B200_BFLOAT16 || dtype == NT_B200_FLOAT32;
}

inline bool is_half_dtype(int dtype) {
  return dtype == NT_B200_FLOAT16 || dtype == NT_B200_BFLOAT16;
}

// Operand dtypes of the contraction programs (matmul, addmm).
inline bool is_gemm_in_dtype(int dtype) {
  return is_half_dtype(dtype) || dtype == NT_B200_FLOAT8_E4M3FN || dtype == NT_B200_FLOAT8_E5M2 ||
         dtype == NT_B200_FLOAT32;
}

inline int dtype_size(int dtype) {
  switch (dtype) {
    case NT_B200_FLOAT16:
    case NT_B200_BFLOAT16: return 2;
    case NT_B200_FLOAT32: return 4;
    default: return 0;
  }
}

// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace nt

// Dispatches `body` with `scalar_t` bound to the element type of a float dtype.
#define NT_DISPATCH_FLOAT(dtype, ...)                                   \
  [&]() -> int {                                                        \
    switch (dtype) {                                                    \
      case NT_B200_FLOAT16: { using scalar_t = __half; return __VA_ARGS__(); }        \
      case NT_B200_BFLOAT16: { using scalar_t = __nv_bfloat16; return __VA_ARGS__(); } \
      case NT_B200_FLOAT32: { using scalar_t = float; return __VA_ARGS__(); }         \
      default: return NT_B200_ERR_UNSUPPORTED_DTYPE;                    \
    }                                                                   \
  }()
