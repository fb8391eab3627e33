// Row softmax (the reference's `softmax_kernel`, tests/test_softmax.py:10-27).
//
// The reference program loads each row twice (once for the max, once for the
// exponentials) with one program per row.  Here a row is read from HBM exactly
// once: the fast path keeps the whole row in registers as 128-bit vectors, one
// CTA per row, so traffic is the algorithmic minimum of one read and one write.
// Math is fp32; the result is rounded once to the output dtype.
#pragma once

#include "common.cuh"

namespace nt {
namespace softmax {

template <int THREADS>
__device__ __forceinline__ float block_reduce_max(float v, float *smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  constexpr int WARPS = THREADS / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  float r = lane < WARPS ? smem[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
  __syncthreads();
  return r;
}

template <int THREADS>
__device__ __forceinline__ float block_reduce_sum(float v, float *smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  constexpr int WARPS = THREADS / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  float r = lane < WARPS ? smem[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  __syncthreads();
  return r;
}

template <typename T> __device__ __forceinline__ float fast_exp(float x);
template <> __device__ __forceinline__ float fast_exp<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ float fast_exp<__half>(float x) { return __expf(x); }
template <> __device__ __forceinline__ float fast_exp<__nv_bfloat16>(float x) { return __expf(x); }

// 128-bit vector of 16/sizeof(T) elements.
template <typename T> struct alignas(16) Vec {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

// Register-resident path: each thread owns VPT vectors of the row; rows must be
// contiguous, 16-byte aligned and cols a multiple of the vector width.  Vector j
// of thread t is vector index j*THREADS + t, so each load instruction of a warp
// covers 512 contiguous bytes.
template <typename T, int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS)
rows_in_registers(const T *__restrict__ input, T *__restrict__ output, int64_t rows,
                  int64_t cols, int64_t in_row_stride, int64_t out_row_stride) {
  using V = Vec<T>;
  constexpr int E = V::N;
  __shared__ float red[32];
  const int64_t nvec = cols / E;
  wait_prior_grid();
  allow_dependent_launch();
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const V *src = reinterpret_cast<const V *>(input + row * in_row_stride);
    V *dst = reinterpret_cast<V *>(output + row * out_row_stride);
    float x[VPT][E];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t idx = (int64_t)j * THREADS + threadIdx.x;
      if (idx < nvec) {
        V vec;
        *reinterpret_cast<int4 *>(&vec) = __ldcs(reinterpret_cast<const int4 *>(src + idx));
#pragma unroll
        for (int e = 0; e < E; ++e) {
          x[j][e] = to_f(vec.v[e]);
          m = fmaxf(m, x[j][e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) x[j][e] = -INFINITY;
      }
    }
    m = block_reduce_max<THREADS>(m, red);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        x[j][e] = fast_exp<T>(x[j][e] - m);
        s += x[j][e];
      }
    }
    s = block_reduce_sum<THREADS>(s, red);
    const float inv = 1.f / s;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t idx = (int64_t)j * THREADS + threadIdx.x;
      if (idx < nvec) {
        V vec;
#pragma unroll
        for (int e = 0; e < E; ++e) vec.v[e] = from_f<T>(x[j][e] * inv);
        __stcs(reinterpret_cast<int4 *>(dst + idx), *reinterpret_cast<int4 *>(&vec));
      }
    }
  }
}

// rows_in_registers for a grid of at most the resident CTAs, each taking
// several rows: a CTA loads its next row while it reduces and writes the
// current one (the same arithmetic, so the same results).
template <typename T, int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS)
rows_prefetched(const T *__restrict__ input, T *__restrict__ output, int64_t rows, int64_t cols,
                int64_t in_row_stride, int64_t out_row_stride) {
  using V = Vec<T>;
  constexpr int E = V::N;
  __shared__ float red[32];
  const int64_t nvec = cols / E;
  wait_prior_grid();
  allow_dependent_launch();
  int4 raw[VPT];
  int64_t row = blockIdx.x;
  if (row < rows) {
    const V *src = reinterpret_cast<const V *>(input + row * in_row_stride);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t idx = (int64_t)j * THREADS + threadIdx.x;
      raw[j] = idx < nvec ? __ldcs(reinterpret_cast<const int4 *>(src + idx)) : make_int4(0, 0, 0, 0);
    }
  }
  for (; row < rows; row += gridDim.x) {
    V *dst = reinterpret_cast<V *>(output + row * out_row_stride);
    float x[VPT][E];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t idx = (int64_t)j * THREADS + threadIdx.x;
      if (idx < nvec) {
        V vec;
        *reinterpret_cast<int4 *>(&vec) = raw[j];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          x[j][e] = to_f(vec.v[e]);
          m = fmaxf(m, x[j][e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) x[j][e] = -INFINITY;
      }
    }
    const int64_t next = row + gridDim.x;
    if (next < rows) {
      const V *src = reinterpret_cast<const V *>(input + next * in_row_stride);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int64_t idx = (int64_t)j * THREADS + threadIdx.x;
        raw[j] = idx < nvec ? __ldcs(reinterpret_cast<const int4 *>(src + idx)) : make_int4(0, 0, 0, 0);
      }
    }
    m = block_reduce_max<THREADS>(m, red);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        x[j][e] = fast_exp<T>(x[j][e] - m);
        s += x[j][e];
      }
    }
    s = block_reduce_sum<THREADS>(s, red);
    const float inv = 1.f / s;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t idx = (int64_t)j * THREADS + threadIdx.x;
      if (idx < nvec) {
        V vec;
#pragma unroll
        for (int e = 0; e < E; ++e) vec.v[e] = from_f<T>(x[j][e] * inv);
        __stcs(reinterpret_cast<int4 *>(dst + idx), *reinterpret_cast<int4 *>(&vec));
      }
    }
  }
}

// Unit column stride, any row length and alignment: the row in registers as
// EPT scalars per thread (element j * THREADS + t), loaded and stored with
// coalesced scalar accesses, so a row is still read from HBM once.
template <typename T, int THREADS, int EPT>
__global__ void __launch_bounds__(THREADS)
rows_in_registers_scalar(const T *__restrict__ input, T *__restrict__ output, int64_t rows, int64_t cols,
                         int64_t in_row_stride, int64_t out_row_stride) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T *src = input + row * in_row_stride;
    T *dst = output + row * out_row_stride;
    float x[EPT];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const int64_t c = (int64_t)j * THREADS + threadIdx.x;
      x[j] = c < cols ? to_f(__ldcs(src + c)) : -INFINITY;
      m = fmaxf(m, x[j]);
    }
    m = block_reduce_max<THREADS>(m, red);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      x[j] = fast_exp<T>(x[j] - m);
      s += x[j];
    }
    s = block_reduce_sum<THREADS>(s, red);
    const float inv = 1.f / s;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const int64_t c = (int64_t)j * THREADS + threadIdx.x;
      if (c < cols) __stcs(dst + c, from_f<T>(x[j] * inv));
    }
  }
}

// General path for any strides and lengths: three passes over the row with
// scalar loads (the second and third hit L2 for rows that fit there).
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
rows_strided(const T *__restrict__ input, T *__restrict__ output, int64_t rows, int64_t cols,
             int64_t isr, int64_t isc, int64_t osr, int64_t osc) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T *src = input + row * isr;
    T *dst = output + row * osr;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < cols; i += THREADS) m = fmaxf(m, to_f(src[i * isc]));
    m = block_reduce_max<THREADS>(m, red);
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < cols; i += THREADS) s += fast_exp<T>(to_f(src[i * isc]) - m);
    s = block_reduce_sum<THREADS>(s, red);
    const float inv = 1.f / s;
    for (int64_t i = threadIdx.x; i < cols; i += THREADS)
      dst[i * osc] = from_f<T>(fast_exp<T>(to_f(src[i * isc]) - m) * inv);
  }
}

template <typename T, int THREADS, int VPT>
inline void launch_regs(const T *in, T *out, int64_t rows, int64_t cols, int64_t isr, int64_t osr,
                        cudaStream_t stream) {
  // Up to four rows per resident CTA (such as one GPU's shard of a split
  // batch): a grid of at most the CTAs that fit on the GPU at once (per
  // device, found on first use), each prefetching its next row.  More rows:
  // one CTA per row.
  static std::atomic<int> resident[64] = {};
  int device = 0;
  cudaGetDevice(&device);
  int per_sm = (device >= 0 && device < 64) ? resident[device].load(std::memory_order_relaxed) : 0;
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rows_prefetched<T, THREADS, VPT>, THREADS,
                                                      0) != cudaSuccess ||
        per_sm <= 0) {
      cudaGetLastError();
      per_sm = 1;
    }
    if (device >= 0 && device < 64) resident[device].store(per_sm, std::memory_order_relaxed);
  }
  const int64_t cap = (int64_t)per_sm * sm_count();
  if (rows <= 4 * cap) {
    const int64_t grid = rows < cap ? rows : cap;
    launch_overlapped(rows_prefetched<T, THREADS, VPT>, dim3((unsigned)grid), dim3(THREADS), 0, stream, in,
                      out, rows, cols, isr, osr);
  } else {
    const int64_t grid = rows < (1 << 30) ? rows : (1 << 30);
    launch_overlapped(rows_in_registers<T, THREADS, VPT>, dim3((unsigned)grid), dim3(THREADS), 0, stream, in,
                      out, rows, cols, isr, osr);
  }
}

template <typename T>
int run(const void *input, void *output, int64_t rows, int64_t cols, int64_t isr, int64_t isc,
        int64_t osr, int64_t osc, cudaStream_t stream) {
  const T *in = static_cast<const T *>(input);
  T *out = static_cast<T *>(output);
  constexpr int E = Vec<T>::N;
  const bool aligned = isc == 1 && osc == 1 && (cols % E) == 0 && (isr % E) == 0 &&
                       (osr % E) == 0 && (reinterpret_cast<uintptr_t>(input) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(output) % 16) == 0;
  const int64_t nvec = cols / E;
  if (aligned && nvec <= 128 * 4) {
    if (nvec <= 32) launch_regs<T, 32, 1>(in, out, rows, cols, isr, osr, stream);
    else if (nvec <= 128) launch_regs<T, 128, 1>(in, out, rows, cols, isr, osr, stream);
    else if (nvec <= 256) launch_regs<T, 128, 2>(in, out, rows, cols, isr, osr, stream);
    else launch_regs<T, 128, 4>(in, out, rows, cols, isr, osr, stream);
  } else if (aligned && nvec <= 256 * 8) {
    if (nvec <= 256 * 4) launch_regs<T, 256, 4>(in, out, rows, cols, isr, osr, stream);
    else launch_regs<T, 256, 8>(in, out, rows, cols, isr, osr, stream);
  } else if (isc == 1 && osc == 1 && cols <= 256 * 16) {
    const int64_t grid = rows < (1 << 30) ? rows : (1 << 30);
    if (cols <= 128 * 4)
      rows_in_registers_scalar<T, 128, 4><<<(unsigned)grid, 128, 0, stream>>>(in, out, rows, cols, isr, osr);
    else if (cols <= 256 * 4)
      rows_in_registers_scalar<T, 256, 4><<<(unsigned)grid, 256, 0, stream>>>(in, out, rows, cols, isr, osr);
    else if (cols <= 256 * 8)
      rows_in_registers_scalar<T, 256, 8><<<(unsigned)grid, 256, 0, stream>>>(in, out, rows, cols, isr, osr);
    else
      rows_in_registers_scalar<T, 256, 16><<<(unsigned)grid, 256, 0, stream>>>(in, out, rows, cols, isr, osr);
  } else {
    const int64_t grid = rows < (1 << 30) ? rows : (1 << 30);
    rows_strided<T, 256><<<(unsigned)grid, 256, 0, stream>>>(in, out, rows, cols, isr, isc, osr, osc);
  }
  return launch_status();
}

}  // namespace softmax
}  // namespace nt

extern "C" int nt_b200_softmax(const void *input, void *output, int64_t rows, int64_t cols,
                               int64_t input_stride_row, int64_t input_stride_col,
                               int64_t output_stride_row, int64_t output_stride_col, int dtype,
                               void *stream) {
  if (rows < 0 || cols < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_float_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (rows == 0 || cols == 0) return 0;
  if (input == nullptr || output == nullptr) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return NT_DISPATCH_FLOAT(dtype, [&] {
    return nt::softmax::run<scalar_t>(input, output, rows, cols, input_stride_row, input_stride_col,
                                      output_stride_row, output_stride_col, s);
  });
}
