// Elementwise programs of the reference: add (tests/test_add.py:9-24), pow
// (tests/test_pow.py:10-31) and dropout (tests/test_dropout.py:12-29).
//
// Contiguous operands take a grid-stride path with 128-bit loads and stores
// (one vector of 16/sizeof(T) elements per thread per iteration); any other
// strides take a scalar grid-stride path.  Grids are sized to a multiple of the
// SM count.
#pragma once

#include <type_traits>

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
  wait_prior_grid();  // launched as a programmatic dependent (launch_overlapped)
  allow_dependent_launch();
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

// ---------------------------------------------------------------- fp16 pow
// pow on fp16 operands with the result of the fp32 path, RN_fp16(powf(x, y)),
// for every pair of fp16 inputs (the GPU tests compare all 2^32 pairs), at a
// fraction of powf's instruction count.
//
// x^y = 2^(y log2 |x|), with log2 |x| for every fp16 bit pattern of |x| from a
// 32768-entry table in shared memory (128 KB: one CTA of 1024 threads per SM)
// built at kernel start: log2(1 + f/1024) in double precision for the 1024
// fractions f, then e + that, rounded once to fp32, for every exponent e
// (subnormal x normalised first); the zero, inf and NaN entries are NaN.
// r = ex2.approx(y T[|x|]) is within a few fp32 ulps of |x|^y, and so is
// powf's result, so the two round to different fp16 values only if an fp16
// rounding boundary lies between them.  An element is computed with powf
// instead when
//   - r lies within kPowWindow fp32 ulps of a midpoint between neighbouring
//     fp16 values (the exact midpoints, such as 63^2 = 3969, among them; for r
//     in the fp16 range these are the r whose 13 bits below the fp16 fraction
//     are near 0x1000, 65520 included),
//   - r lies in [2^-25.5, 2^-14), where fp16 rounds on its subnormal grid, or
//   - r is NaN (x zero, inf or NaN; y NaN; 1^inf).
// Larger r rounds to inf and smaller r to zero, as powf's result does.  For
// negative x the sign follows y: NaN unless y is an integer, negative for odd
// y.  A window of 16 ulps leaves no pair of fp16 inputs with a result
// different from the fp32 path (checked exhaustively on the B200).
// The elements sent to powf are queued per warp and computed 32 at a time, so
// a rare one costs its warp 1/32 of a powf pass instead of a divergent pass.
constexpr uint32_t kPowWindow = 16;
constexpr uint32_t kPowBandLo = 0x32B50000u;  // 2^-25.5, rounded down
constexpr uint32_t kPowBandHi = 0x387fffc0u;  // 2^-14 (1 - 2^-17)
constexpr int kPowThreads = 1024;
constexpr int kPowQueue = 64;  // deferred elements per warp

struct PowHalfShared {
  float log2_abs[32768];                          // log2 of |x| by fp16 bit pattern
  int64_t queue[kPowThreads / 32][kPowQueue];     // deferred element indices per warp
  int fill[kPowThreads / 32];                     // places taken in a warp's queue this step
};

__device__ __forceinline__ void build_pow_table(PowHalfShared &sh) {
  float2 *frac = reinterpret_cast<float2 *>(&sh.queue[0][0]);  // log2(1 + f/1024) as hi + lo, 8 KB
  for (int f = threadIdx.x; f < 1024; f += blockDim.x) {
    const double l = log2(1.0 + f * (1.0 / 1024.0));
    const float hi = static_cast<float>(l);
    frac[f] = make_float2(hi, static_cast<float>(l - static_cast<double>(hi)));
  }
  __syncthreads();
  for (int xb = threadIdx.x; xb < 32768; xb += blockDim.x) {
    const int E = xb >> 10, f = xb & 0x3ff;
    float v;
    if (E == 31 || xb == 0) {
      v = __int_as_float(0x7fffffff);  // zero, inf, NaN: powf
    } else {
      int e = E - 15, ff = f;
      if (E == 0) {  // subnormal: f 2^-24 = 2^(k - 24) (f / 2^k)
        const int k = 31 - __clz(f);
        e = k - 24;
        ff = (f << (10 - k)) & 0x3ff;
      }
      const float2 l = frac[ff];
      v = static_cast<float>(static_cast<double>(e) + static_cast<double>(l.x) + static_cast<double>(l.y));
    }
    sh.log2_abs[xb] = v;
  }
  if (threadIdx.x < kPowThreads / 32) sh.fill[threadIdx.x] = 0;
  __syncthreads();  // the fraction table's space becomes the queues
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// r ~ |x|^y; true when the element must be computed with powf
__device__ __forceinline__ bool pow_half_abs(uint32_t xb, uint32_t yb, const PowHalfShared &sh, float &r) {
  const float y = __half2float(__ushort_as_half(static_cast<unsigned short>(yb)));
  r = ex2_approx(y * sh.log2_abs[xb & 0x7fffu]);
  const uint32_t rb = __float_as_uint(r);
  const bool band = (rb - kPowBandLo) < (kPowBandHi - kPowBandLo);
  const bool nan = rb > 0x7f800000u;
  const bool near = ((rb + (kPowWindow - 0x1000u)) & 0x1fffu) <= 2u * kPowWindow;
  return band | nan | near;
}

// x^y from r = |x|^y for negative x
__device__ __forceinline__ float pow_half_sign(uint32_t xb, uint32_t yb, float r) {
  if (!(xb & 0x8000u)) return r;
  const float y = __half2float(__ushort_as_half(static_cast<unsigned short>(yb)));
  if (truncf(y) != y) return __int_as_float(0x7fffffff);
  const bool odd = fabsf(y) < 2048.f && (__float2int_rz(y) & 1);
  return odd ? -r : r;
}

__device__ __forceinline__ void pow_half_slow(const __half *a, const __half *b, __half *out, int64_t k) {
  out[k] = __float2half_rn(PowOp{}(__half2float(a[k]), __half2float(b[k])));
}

// Persistent: one CTA per SM; each warp takes two 32-vector blocks (8 elements
// a lane) per step, `stride` vectors apart.
__global__ void __launch_bounds__(kPowThreads, 1)
pow_half_kernel(const __half *__restrict__ a, const __half *__restrict__ b, __half *__restrict__ out,
                int64_t nvec) {
  extern __shared__ __align__(16) uint8_t pow_smem[];
  PowHalfShared &sh = *reinterpret_cast<PowHalfShared *>(pow_smem);
  build_pow_table(sh);  // no global memory: runs beside the previous kernel's tail
  wait_prior_grid();    // launched as a programmatic dependent (launch_overlapped)
  allow_dependent_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t *queue = sh.queue[warp];
  using V = Vec<__half>;
  const V *va = reinterpret_cast<const V *>(a);
  const V *vb = reinterpret_cast<const V *>(b);
  V *vo = reinterpret_cast<V *>(out);
  int count = 0;  // queued elements of this warp (the same in every lane)
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = blockIdx.x * (int64_t)blockDim.x + warp * 32; base < nvec; base += 2 * stride) {
    int64_t idx[2];
    V x[2], y[2];
    uint32_t slow[2] = {0u, 0u};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      idx[h] = base + h * stride + lane;
      if (idx[h] < nvec) {
        *reinterpret_cast<int4 *>(&x[h]) = __ldcs(reinterpret_cast<const int4 *>(va + idx[h]));
        *reinterpret_cast<int4 *>(&y[h]) = __ldcs(reinterpret_cast<const int4 *>(vb + idx[h]));
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (idx[h] >= nvec) continue;
      float r[V::N];
#pragma unroll
      for (int e = 0; e < V::N; ++e)
        slow[h] |= static_cast<uint32_t>(
                       pow_half_abs(__half_as_ushort(x[h].v[e]), __half_as_ushort(y[h].v[e]), sh, r[e]))
                   << e;
      const uint32_t *xw = reinterpret_cast<const uint32_t *>(&x[h]);
      if ((xw[0] | xw[1] | xw[2] | xw[3]) & 0x80008000u) {  // a negative x among the eight
#pragma unroll
        for (int e = 0; e < V::N; ++e)
          r[e] = pow_half_sign(__half_as_ushort(x[h].v[e]), __half_as_ushort(y[h].v[e]), r[e]);
      }
      V z;
#pragma unroll
      for (int e = 0; e < V::N; e += 2) *reinterpret_cast<__half2 *>(&z.v[e]) = __floats2half2_rn(r[e], r[e + 1]);
      __stcs(reinterpret_cast<int4 *>(vo + idx[h]), *reinterpret_cast<int4 *>(&z));
    }
    // queue this step's slow elements (lanes take consecutive places from
    // the warp's fill counter, in any order); compute 32 of them once 32 are
    // queued
    const int n = __popc(slow[0]) + __popc(slow[1]);
    const int total = (int)__reduce_add_sync(0xffffffffu, (unsigned)n);
    if (total != 0) {
      if (count + total > kPowQueue) {  // no room: compute what is queued first
        for (int q = lane; q < count; q += 32) pow_half_slow(a, b, out, queue[q]);
        count = 0;
        __syncwarp();
      }
      if (total > kPowQueue) {  // more than a queue's worth: every lane its own
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t bits = slow[h];
          while (bits) {
            const int e = __ffs(bits) - 1;
            bits &= bits - 1;
            pow_half_slow(a, b, out, idx[h] * V::N + e);
          }
        }
      } else {
        int pos = count;
        if (n != 0) pos += atomicAdd(&sh.fill[warp], n);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t bits = slow[h];
          while (bits) {
            const int e = __ffs(bits) - 1;
            bits &= bits - 1;
            queue[pos++] = idx[h] * V::N + e;
          }
        }
        __syncwarp();  // queue entries and this step's vector stores ordered before the powf pass
        if (lane == 0) sh.fill[warp] = 0;
        count += total;
        __syncwarp();
        while (count >= 32) {
          pow_half_slow(a, b, out, queue[count - 32 + lane]);
          count -= 32;
          __syncwarp();
        }
      }
    }
  }
  for (int q = lane; q < count; q += 32) pow_half_slow(a, b, out, queue[q]);
}

template <typename T>
__global__ void dropout_vec(const T *__restrict__ in, T *__restrict__ out, int64_t nvec, float p,
                            uint32_t key_lo, uint32_t key_hi) {
  using V = Vec<T>;
  const V *vi = reinterpret_cast<const V *>(in);
  V *vo = reinterpret_cast<V *>(out);
  const float keep = 1.f - p;
  const float inv_keep = __frcp_rn(keep);
  wait_prior_grid();  // launched as a programmatic dependent (launch_overlapped)
  allow_dependent_launch();
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
    if (nvec > 0) {
      const int e = launch_overlapped(binary_vec<T, Op>, dim3(grid_for(nvec, THREADS)), dim3(THREADS), 0, stream, pa,
                                      pb, po, nvec, op);
      if (e != 0) return launch_status();  // the launch's error, cleared
    }
    done = nvec * Vec<T>::N;
  }
  if (done < size)
    binary_strided<T, Op><<<grid_for(size - done, THREADS), THREADS, 0, stream>>>(pa, pb, po, size, sa, sb,
                                                                                 so, done, op);
  return launch_status();
}

// pow: contiguous fp16 operands of 2^20 elements and more take
// pow_half_kernel on their vector part (same results as the powf path,
// element for element; below that size its table build costs more than it
// saves); every other case is run_binary.
template <typename T>
int run_pow(const void *a, const void *b, void *out, int64_t size, int64_t sa, int64_t sb, int64_t so,
            cudaStream_t stream) {
  if constexpr (std::is_same<T, __half>::value) {
    constexpr int THREADS = 256;
    if (size >= (1 << 20) && sa == 1 && sb == 1 && so == 1 && vec_ok<T>(a) && vec_ok<T>(b) && vec_ok<T>(out)) {
      const __half *pa = static_cast<const __half *>(a);
      const __half *pb = static_cast<const __half *>(b);
      __half *po = static_cast<__half *>(out);
      const int64_t nvec = size / Vec<T>::N;
      const cudaError_t e = smem_optin<pow_half_kernel>((int)sizeof(PowHalfShared));
      if (e != cudaSuccess) return (int)e;
      const int le = launch_overlapped(pow_half_kernel, dim3(sm_count()), dim3(kPowThreads), sizeof(PowHalfShared),
                                       stream, pa, pb, po, nvec);
      if (le != 0) return launch_status();  // the launch's error, cleared
      const int64_t done = nvec * Vec<T>::N;
      if (done < size)
        binary_strided<T, PowOp><<<grid_for(size - done, THREADS), THREADS, 0, stream>>>(pa, pb, po, size, 1, 1, 1,
                                                                                      done, PowOp{});
      return launch_status();
    }
  }
  return run_binary<T>(a, b, out, size, sa, sb, so, PowOp{}, stream);
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
    if (nvec > 0) {
      const int e = launch_overlapped(dropout_vec<T>, dim3(grid_for(nvec, THREADS)), dim3(THREADS), 0, stream, pi, po,
                                      nvec, p, key_lo, key_hi);
      if (e != 0) return launch_status();  // the launch's error, cleared
    }
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
    return nt::elementwise::run_pow<scalar_t>(input, exponent, output, size, input_stride, exponent_stride,
                                              output_stride, s);
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
