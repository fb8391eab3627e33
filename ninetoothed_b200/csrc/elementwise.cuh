// Elementwise programs of the reference: add (tests/test_add.py:9-24), pow
// (tests/test_pow.py:10-31) and dropout (tests/test_dropout.py:12-29).
//
// Contiguous operands take a grid-stride path with 128-bit loads and stores
// (one vector of 16/sizeof(T) elements per thread per iteration); any other
// strides take a scalar grid-stride path.  Grids are sized to a multiple of the
// SM count.
#pragma once

#include "common.cuh"

namespace nt {
namespace elementwise {

// ---------------------------------------------------------------- Philox
// Philox4x32 with 10 rounds (Salmon et al., "Parallel random numbers: as easy
// as 1, 2, 3", SC'11), keyed by the 64-bit seed split into (lo, hi) words and
// run on the counter (offset, 0, 0, 0).  This is the generator behind Triton's
// `tl.rand(seed, offset)` (triton/language/random.py, `philox_impl`,
// `randint4x`, `uint_to_uniform_float`), which the reference dropout calls.
// Each round's two 32 x 32 -> 64-bit products are taken whole (high and low
// words from one wide multiply), and the last round computes only word 0.
__device__ __forceinline__ uint32_t philox_first_word(uint32_t c0, uint32_t key_lo, uint32_t key_hi) {
  uint32_t c1 = 0, c2 = 0, c3 = 0;
  uint32_t k0 = key_lo, k1 = key_hi;
#pragma unroll
  for (int round = 0; round < 9; ++round) {
    const uint64_t w1 = (uint64_t)0xCD9E8D57u * c2;
    const uint64_t w0 = (uint64_t)0xD2511F53u * c0;
    c0 = (uint32_t)(w1 >> 32) ^ c1 ^ k0;
    c2 = (uint32_t)(w0 >> 32) ^ c3 ^ k1;
    c1 = (uint32_t)w1;
    c3 = (uint32_t)w0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return __umulhi(0xCD9E8D57u, c2) ^ c1 ^ k0;
}

// x / keep rounded once to fp32, for 16-bit-float x (normal in fp32) and keep
// in (0, 1]: with y = RN(1 / keep), q0 = RN(x * y) is within an ulp of x / keep,
// r = x - q0 * keep is exact (one FMA), and RN(q0 + r * y) is the correctly
// rounded quotient (Markstein's theorem, "Computation of elementary functions
// on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990), so the
// result equals an IEEE division.  Wider inputs keep the plain division.
template <typename T>
__device__ __forceinline__ float scale_kept(float x, float keep, float inv_keep) {
  if constexpr (sizeof(T) == 2 && Elem<T>::is_f16) {
    const float q0 = x * inv_keep;
    const float r = __fmaf_rn(-q0, keep, x);
    return __fmaf_rn(r, inv_keep, q0);
  } else {
    return __fdiv_rn(x, keep);
  }
}

// Maps a 32-bit word to [0, 1): reinterpret as int32, fold negatives with
// -x - 1, convert to fp32 (round to nearest) and scale by 2^-31.
__device__ __forceinline__ float uniform_from_word(uint32_t word) {
  int32_t x = static_cast<int32_t>(word);
  x = x < 0 ? -x - 1 : x;
  return __int2float_rn(x) * 4.6566127342e-10f;
}

struct AddOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return a + b; }
};
struct PowOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return powf(a, b); }
};

template <typename T> struct alignas(16) Vec {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

template <typename T, typename Op>
__global__ void binary_vec(const T *__restrict__ a, const T *__restrict__ b, T *__restrict__ out,
                           int64_t nvec, Op op) {
  using V = Vec<T>;
  const V *va = reinterpret_cast<const V *>(a);
  const V *vb = reinterpret_cast<const V *>(b);
  V *vo = reinterpret_cast<V *>(out);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    V x, y, z;
    *reinterpret_cast<int4 *>(&x) = __ldcs(reinterpret_cast<const int4 *>(va + i));
    *reinterpret_cast<int4 *>(&y) = __ldcs(reinterpret_cast<const int4 *>(vb + i));
#pragma unroll
    for (int e = 0; e < V::N; ++e) z.v[e] = from_f<T>(op(to_f(x.v[e]), to_f(y.v[e])));
    __stcs(reinterpret_cast<int4 *>(vo + i), *reinterpret_cast<int4 *>(&z));
  }
}

template <typename T, typename Op>
__global__ void binary_strided(const T *__restrict__ a, const T *__restrict__ b, T *__restrict__ out,
                               int64_t size, int64_t sa, int64_t sb, int64_t so, int64_t start, Op op) {
  for (int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < size;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i * so] = from_f<T>(op(to_f(a[i * sa]), to_f(b[i * sb])));
}

template <typename T>
__global__ void dropout_vec(const T *__restrict__ in, T *__restrict__ out, int64_t nvec, float p,
                            uint32_t key_lo, uint32_t key_hi) {
  using V = Vec<T>;
  const V *vi = reinterpret_cast<const V *>(in);
  V *vo = reinterpret_cast<V *>(out);
  const float keep = 1.f - p;
  const float inv_keep = __frcp_rn(keep);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    V x, z;
    *reinterpret_cast<int4 *>(&x) = __ldcs(reinterpret_cast<const int4 *>(vi + i));
#pragma unroll
    for (int e = 0; e < V::N; ++e) {
      const uint32_t offset = static_cast<uint32_t>(i * V::N + e);
      const float r = uniform_from_word(philox_first_word(offset, key_lo, key_hi));
      z.v[e] = from_f<T>(r > p ? scale_kept<T>(to_f(x.v[e]), keep, inv_keep) : 0.f);
    }
    __stcs(reinterpret_cast<int4 *>(vo + i), *reinterpret_cast<int4 *>(&z));
  }
}

template <typename T>
__global__ void dropout_strided(const T *__restrict__ in, T *__restrict__ out, int64_t size,
                                int64_t si, int64_t so, int64_t start, float p, uint32_t key_lo,
                                uint32_t key_hi) {
  const float keep = 1.f - p;
  for (int64_t i = start + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < size;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float r = uniform_from_word(philox_first_word(static_cast<uint32_t>(i), key_lo, key_hi));
    out[i * so] = from_f<T>(r > p ? __fdiv_rn(to_f(in[i * si]), keep) : 0.f);
  }
}

inline unsigned grid_for(int64_t work, int threads) {
  const int64_t cap = (int64_t)sm_count() * 8;  // 8 resident CTAs of 256 threads per SM
  int64_t g = (work + threads - 1) / threads;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

template <typename T>
inline bool vec_ok(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) % 16) == 0;
}

template <typename T, typename Op>
int run_binary(const void *a, const void *b, void *out, int64_t size, int64_t sa, int64_t sb,
               int64_t so, Op op, cudaStream_t stream) {
  constexpr int THREADS = 256;
  const T *pa = static_cast<const T *>(a);
  const T *pb = static_cast<const T *>(b);
  T *po = static_cast<T *>(out);
  int64_t done = 0;
  if (sa == 1 && sb == 1 && so == 1 && vec_ok<T>(a) && vec_ok<T>(b) && vec_ok<T>(out)) {
    const int64_t nvec = size / Vec<T>::N;
    if (nvec > 0) binary_vec<T, Op><<<grid_for(nvec, THREADS), THREADS, 0, stream>>>(pa, pb, po, nvec, op);
    done = nvec * Vec<T>::N;
  }
  if (done < size)
    binary_strided<T, Op><<<grid_for(size - done, THREADS), THREADS, 0, stream>>>(pa, pb, po, size, sa, sb,
                                                                                 so, done, op);
  return launch_status();
}

template <typename T>
int run_dropout(const void *in, void *out, int64_t size, int64_t si, int64_t so, float p, int64_t seed,
                cudaStream_t stream) {
  constexpr int THREADS = 256;
  // The seed is widened to 64 bits and split into key words (lo, hi).
  const uint64_t s = static_cast<uint64_t>(seed);
  const uint32_t key_lo = static_cast<uint32_t>(s & 0xffffffffu);
  const uint32_t key_hi = static_cast<uint32_t>(s >> 32);
  const T *pi = static_cast<const T *>(in);
  T *po = static_cast<T *>(out);
  int64_t done = 0;
  if (si == 1 && so == 1 && vec_ok<T>(in) && vec_ok<T>(out)) {
    const int64_t nvec = size / Vec<T>::N;
    if (nvec > 0)
      dropout_vec<T><<<grid_for(nvec, THREADS), THREADS, 0, stream>>>(pi, po, nvec, p, key_lo, key_hi);
    done = nvec * Vec<T>::N;
  }
  if (done < size)
    dropout_strided<T><<<grid_for(size - done, THREADS), THREADS, 0, stream>>>(pi, po, size, si, so, done, p,
                                                                              key_lo, key_hi);
  return launch_status();
}

}  // namespace elementwise
}  // namespace nt

extern "C" int nt_b200_add(const void *lhs, const void *rhs, void *output, int64_t size, int64_t lhs_stride,
                           int64_t rhs_stride, int64_t output_stride, int dtype, void *stream) {
  if (size < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_float_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (size == 0) return 0;
  if (!lhs || !rhs || !output) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return NT_DISPATCH_FLOAT(dtype, [&] {
    return nt::elementwise::run_binary<scalar_t>(lhs, rhs, output, size, lhs_stride, rhs_stride,
                                                 output_stride, nt::elementwise::AddOp{}, s);
  });
}

extern "C" int nt_b200_pow(const void *input, const void *exponent, void *output, int64_t size,
                           int64_t input_stride, int64_t exponent_stride, int64_t output_stride, int dtype,
                           void *stream) {
  if (size < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_float_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (size == 0) return 0;
  if (!input || !exponent || !output) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return NT_DISPATCH_FLOAT(dtype, [&] {
    return nt::elementwise::run_binary<scalar_t>(input, exponent, output, size, input_stride, exponent_stride,
                                                 output_stride, nt::elementwise::PowOp{}, s);
  });
}

extern "C" int nt_b200_dropout(const void *input, float p, int64_t seed, void *output, int64_t size,
                               int64_t input_stride, int64_t output_stride, int dtype, void *stream) {
  if (size < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_float_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (size == 0) return 0;
  if (!input || !output) return NT_B200_ERR_INVALID_ARGUMENT;
  if (size > (int64_t)0xffffffffLL) return NT_B200_ERR_INVALID_ARGUMENT;  // 32-bit Philox counter
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return NT_DISPATCH_FLOAT(dtype, [&] {
    return nt::elementwise::run_dropout<scalar_t>(input, output, size, input_stride, output_stride, p, seed, s);
  });
}
