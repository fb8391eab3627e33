// General-layout CUDA-core paths for the contraction programs (matmul, addmm,
// conv2d) and attention.  They take any element strides and any sizes and are
// used when an operand layout does not meet the TMA rules of the tensor-core
// kernels (16-byte aligned base and row strides, unit inner stride).  They
// compute the same expression as the tensor-core kernels: fp32 accumulation in
// ascending k, then the application's cast chain.
#pragma once

#include "common.cuh"

namespace nt {
namespace simt {

// ------------------------------------------------------------ operand access
template <typename T> struct MatrixA {  // A[m, k] of a row/col strided matrix
  const T *p;
  int64_t sm, sk;
  __device__ __forceinline__ float operator()(int64_t m, int64_t k) const { return to_f(p[m * sm + k * sk]); }
};
template <typename T> struct MatrixB {  // B[k, n]
  const T *p;
  int64_t sk, sn;
  __device__ __forceinline__ float operator()(int64_t k, int64_t n) const { return to_f(p[k * sk + n * sn]); }
};

// im2col view of an NCHW input: row m = (image, p, q) of the output, column
// k = (c, r, s) in the order the reference arrangement flattens the filter tile.
template <typename T> struct Im2col {
  const T *p;
  int64_t C, H, W, R, S, P, Q, ph, pw;
  int64_t sn, sc, sh, sw;
  __device__ __forceinline__ float operator()(int64_t m, int64_t k) const {
    const int64_t q = m % Q, t = m / Q, pp = t % P, img = t / P;
    const int64_t s = k % S, t2 = k / S, r = t2 % R, c = t2 / R;
    const int64_t y = pp + r - ph, x = q + s - pw;
    if (y < 0 || y >= H || x < 0 || x >= W) return 0.f;
    return to_f(p[img * sn + c * sc + y * sh + x * sw]);
  }
};
template <typename T> struct FilterB {  // B[k, n] = filter[n, c, r, s]
  const T *p;
  int64_t R, S, sk_, sc, sr, ss;
  __device__ __forceinline__ float operator()(int64_t k, int64_t n) const {
    const int64_t s = k % S, t = k / S, r = t % R, c = t / R;
    return to_f(p[n * sk_ + c * sc + r * sr + s * ss]);
  }
};

// ------------------------------------------------------------ epilogues
template <typename TO> struct StoreMatmul {  // out = cast_out(cast_f16(acc))
  TO *p;
  int64_t sm, sn;
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float acc) const {
    p[m * sm + n * sn] = from_f<TO>(round_f16(acc));
  }
};
template <typename TI, typename TO> struct StoreAddmm {  // beta*input + alpha*cast_f16(acc), typed
  const TI *in;
  TO *p;
  int64_t ism, isn, sm, sn;
  float beta_t, alpha_h;  // scalars rounded to TI and float16
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float acc) const {
    p[m * sm + n * sn] = from_f<TO>(addmm_value<TI>(beta_t, alpha_h, to_f(in[m * ism + n * isn]), acc));
  }
};
template <typename TO> struct StoreConv {  // row m = (image, p, q) -> NCHW output
  TO *p;
  int64_t P, Q, sn, sk, sh, sw;
  __device__ __forceinline__ void operator()(int64_t m, int64_t n, float acc) const {
    const int64_t q = m % Q, t = m / Q, pp = t % P, img = t / P;
    p[img * sn + n * sk + pp * sh + q * sw] = from_f<TO>(round_f16(acc));
  }
};

// 64x64 output tile per 256-thread CTA, 4x4 outputs per thread, K in steps of 16
// staged through shared memory.  The grid is 1-D over (row tile, column tile).
template <typename LA, typename LB, typename ST>
__global__ void __launch_bounds__(256)
gemm_kernel(LA a, LB b, ST st, int64_t M, int64_t N, int64_t K, int64_t tiles_n) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float as[BK][BM + 1];
  __shared__ float bs[BK][BN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t tile = blockIdx.x;
  const int64_t m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int mm = i / BK, kk = i % BK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      as[kk][mm] = (gm < M && gk < K) ? a(gm, gk) : 0.f;
    }
    for (int i = threadIdx.x; i < BN * BK; i += 256) {
      const int nn = i % BN, kk = i / BN;
      const int64_t gn = n0 + nn, gk = k0 + kk;
      bs[kk][nn] = (gn < N && gk < K) ? b(gk, gn) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = as[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gm = m0 + ty + 16 * i, gn = n0 + tx + 16 * j;
      if (gm < M && gn < N) st(gm, gn, acc[i][j]);
    }
}

template <typename LA, typename LB, typename ST>
inline int launch_gemm(LA a, LB b, ST st, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  const int64_t tiles_n = (N + 63) / 64, tiles_m = (M + 63) / 64;
  const int64_t tiles = tiles_n * tiles_m;
  if (tiles > (1LL << 31) - 1) return NT_B200_ERR_INVALID_ARGUMENT;
  gemm_kernel<LA, LB, ST><<<(unsigned)tiles, 256, 0, stream>>>(a, b, st, M, N, K, tiles_n);
  return launch_status();
}

// ------------------------------------------------------------ attention
struct Strides4 {
  int64_t b, h, s, d;
};

// One warp per query row; keys in blocks of 64 (the lower bound of the
// reference's BLOCK_SIZE_N); the reference application's online softmax
// (tests/test_attention.py:44-70): q' = round(q * round(log2 e)), s = q'.k in
// fp32, masked keys at -inf, m starts at -inf and l at 1, p = exp2(s - m_new)
// rounded to T before p @ v, alpha = exp2(m_old - m_new), o = acc / l.
template <typename T>
__global__ void __launch_bounds__(128)
attention_kernel(const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v, T *__restrict__ o,
                 int64_t B, int64_t H, int64_t SQ, int64_t SK, int64_t D, Strides4 qs, Strides4 ks, Strides4 vs,
                 Strides4 os, int causal, float log2e_rounded) {
  constexpr int BN = 64, DPL = 4;  // head_dim <= 128 = 32 lanes x 4
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= B * H * SQ) return;
  const int64_t qi = row % SQ, bh = row / SQ, hi = bh % H, bi = bh / H;
  const T *qrow = q + bi * qs.b + hi * qs.h + qi * qs.s;
  const T *kbase = k + bi * ks.b + hi * ks.h;
  const T *vbase = v + bi * vs.b + hi * vs.h;
  float qv[DPL], acc[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) {
    const int64_t d = lane + 32 * e;
    qv[e] = d < D ? to_f(from_f<T>(to_f(qrow[d * qs.d]) * log2e_rounded)) : 0.f;
    acc[e] = 0.f;
  }
  float m_i = -INFINITY, l_i = 1.f;
  for (int64_t j0 = 0; j0 < SK; j0 += BN) {
    float sblk[BN];
    float m_blk = -INFINITY;
    for (int j = 0; j < BN; ++j) {
      const int64_t kj = j0 + j;
      float part = 0.f;
      if (kj < SK) {
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
          const int64_t d = lane + 32 * e;
          if (d < D) part = fmaf(qv[e], to_f(kbase[kj * ks.s + d * ks.d]), part);
        }
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o2);
      const bool valid = kj < SK && (!causal || qi >= kj);
      sblk[j] = valid ? part : -INFINITY;
      m_blk = fmaxf(m_blk, sblk[j]);
    }
    const float m_new = fmaxf(m_i, m_blk);
    const float alpha = exp2f(m_i - m_new);
    float l_blk = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[e] *= alpha;
    for (int j = 0; j < BN; ++j) {
      const float p = exp2f(sblk[j] - m_new);
      l_blk += p;
      const int64_t kj = j0 + j;
      if (kj < SK) {
        const float pr = to_f(from_f<T>(p));
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
          const int64_t d = lane + 32 * e;
          if (d < D) acc[e] = fmaf(pr, to_f(vbase[kj * vs.s + d * vs.d]), acc[e]);
        }
      }
    }
    m_i = m_new;
    l_i = l_i * alpha + l_blk;
  }
  T *orow = o + bi * os.b + hi * os.h + qi * os.s;
#pragma unroll
  for (int e = 0; e < DPL; ++e) {
    const int64_t d = lane + 32 * e;
    if (d < D) orow[d * os.d] = from_f<T>(acc[e] / l_i);
  }
}

}  // namespace simt
}  // namespace nt
