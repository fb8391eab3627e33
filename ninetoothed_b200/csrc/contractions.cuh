// C-ABI entry points of the contraction programs: matmul, addmm, conv2d and
// attention.  Each picks the tcgen05 tensor-core kernel when the operands meet
// its layout rules and the general-layout CUDA-core kernel otherwise.
#pragma once

#include "common.cuh"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "attention_tc.cuh"

namespace nt {

template <typename TI, typename TO>
int matmul_simt(const void *a, const void *b, void *c, int64_t M, int64_t N, int64_t K, int64_t sam, int64_t sak,
                int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, cudaStream_t s) {
  simt::MatrixA<TI> A{static_cast<const TI *>(a), sam, sak};
  simt::MatrixB<TI> B{static_cast<const TI *>(b), sbk, sbn};
  simt::StoreMatmul<TO> st{static_cast<TO *>(c), scm, scn};
  return simt::launch_gemm(A, B, st, M, N, K, s);
}

template <typename TI, typename TO>
int addmm_simt(const void *in, const void *a, const void *b, float beta, float alpha, void *c, int64_t M,
               int64_t N, int64_t K, int64_t sim, int64_t sin_, int64_t sam, int64_t sak, int64_t sbk, int64_t sbn,
               int64_t scm, int64_t scn, cudaStream_t s) {
  simt::MatrixA<TI> A{static_cast<const TI *>(a), sam, sak};
  simt::MatrixB<TI> B{static_cast<const TI *>(b), sbk, sbn};
  simt::StoreAddmm<TI, TO> st{static_cast<const TI *>(in), static_cast<TO *>(c), sim, sin_, scm, scn, beta, alpha};
  // beta/alpha arrive already rounded (see nt_b200_addmm)
  return simt::launch_gemm(A, B, st, M, N, K, s);
}

// Dispatches (in_dtype, out_dtype) to a functor templated on both.
template <typename F>
int dispatch_in_out(int in_dtype, int out_dtype, F &&f) {
  auto with_out = [&](auto in_tag) -> int {
    using TI = decltype(in_tag);
    switch (out_dtype) {
      case NT_B200_FLOAT16: return f(TI{}, __half{});
      case NT_B200_BFLOAT16: return f(TI{}, __nv_bfloat16{});
      case NT_B200_FLOAT32: return f(TI{}, float{});
      default: return NT_B200_ERR_UNSUPPORTED_DTYPE;
    }
  };
  switch (in_dtype) {
    case NT_B200_FLOAT16: return with_out(__half{});
    case NT_B200_BFLOAT16: return with_out(__nv_bfloat16{});
    case NT_B200_FLOAT8_E4M3FN: return with_out(__nv_fp8_e4m3{});
    case NT_B200_FLOAT8_E5M2: return with_out(__nv_fp8_e5m2{});
    case NT_B200_FLOAT32: return with_out(float{});  // exact fp32 on the CUDA-core path
    default: return NT_B200_ERR_UNSUPPORTED_DTYPE;
  }
}

}  // namespace nt

extern "C" int nt_b200_matmul(const void *lhs, const void *rhs, void *output, int64_t m, int64_t n, int64_t k,
                              int64_t lhs_stride_row, int64_t lhs_stride_col, int64_t rhs_stride_row,
                              int64_t rhs_stride_col, int64_t output_stride_row, int64_t output_stride_col,
                              int in_dtype, int out_dtype, void *stream) {
  if (m < 0 || n < 0 || k < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_gemm_in_dtype(in_dtype) || !nt::is_float_dtype(out_dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (m == 0 || n == 0) return 0;
  if (!output || (k > 0 && (!lhs || !rhs))) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return nt::dispatch_in_out(in_dtype, out_dtype, [&](auto ti, auto to) -> int {
    using TI = decltype(ti);
    using TO = decltype(to);
    const nt::tc::GemmProblem prob{lhs, rhs, nullptr, output, m, n, k, lhs_stride_row, lhs_stride_col,
                                   rhs_stride_row, rhs_stride_col, 0, 0, output_stride_row, output_stride_col,
                                   0.f, 0.f};
    const int rc = nt::tc::try_gemm<TI, TO, nt::tc::Epilogue::kMatmul>(prob, s);
    if (rc != nt::tc::kNotEligible) return rc;
    return nt::matmul_simt<TI, TO>(lhs, rhs, output, m, n, k, lhs_stride_row, lhs_stride_col, rhs_stride_row,
                                   rhs_stride_col, output_stride_row, output_stride_col, s);
  });
}

extern "C" int nt_b200_addmm(const void *input, const void *mat1, const void *mat2, float beta, float alpha,
                             void *output, int64_t m, int64_t n, int64_t k, int64_t input_stride_row,
                             int64_t input_stride_col, int64_t mat1_stride_row, int64_t mat1_stride_col,
                             int64_t mat2_stride_row, int64_t mat2_stride_col, int64_t output_stride_row,
                             int64_t output_stride_col, int in_dtype, int out_dtype, void *stream) {
  if (m < 0 || n < 0 || k < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_gemm_in_dtype(in_dtype) || !nt::is_float_dtype(out_dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (m == 0 || n == 0) return 0;
  if (!output || !input || (k > 0 && (!mat1 || !mat2))) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return nt::dispatch_in_out(in_dtype, out_dtype, [&](auto ti, auto to) -> int {
    using TI = decltype(ti);
    using TO = decltype(to);
    // Scalars take the dtype of the tensor they multiply (Triton's typing of a
    // scalar argument against a tensor): beta -> TI, alpha -> float16.
    const float beta_t = static_cast<float>(typename nt::ScaleType<TI>::type(beta));
    const float alpha_h = static_cast<float>(__half(alpha));
    beta = beta_t;
    alpha = alpha_h;
    const nt::tc::GemmProblem prob{mat1, mat2, input, output, m, n, k, mat1_stride_row, mat1_stride_col,
                                   mat2_stride_row, mat2_stride_col, input_stride_row, input_stride_col,
                                   output_stride_row, output_stride_col, beta, alpha};
    const int rc = nt::tc::try_gemm<TI, TO, nt::tc::Epilogue::kAddmm>(prob, s);
    if (rc != nt::tc::kNotEligible) return rc;
    return nt::addmm_simt<TI, TO>(input, mat1, mat2, beta, alpha, output, m, n, k, input_stride_row,
                                  input_stride_col, mat1_stride_row, mat1_stride_col, mat2_stride_row,
                                  mat2_stride_col, output_stride_row, output_stride_col, s);
  });
}

extern "C" int nt_b200_conv2d(const void *input, const void *filter, void *output, int64_t n, int64_t c, int64_t h,
                              int64_t w, int64_t k, int64_t r, int64_t s, int64_t pad_h, int64_t pad_w,
                              const int64_t *input_strides, const int64_t *filter_strides,
                              const int64_t *output_strides, void *workspace, int64_t workspace_bytes, int dtype,
                              void *stream) {
  if (n < 0 || c < 0 || h < 0 || w < 0 || k < 0 || r <= 0 || s <= 0 || pad_h < 0 || pad_w < 0)
    return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_half_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  const int64_t P = h + 2 * pad_h - r + 1, Q = w + 2 * pad_w - s + 1;
  if (P < 0 || Q < 0) return NT_B200_ERR_SHAPE_MISMATCH;
  if (n == 0 || k == 0 || P == 0 || Q == 0) return 0;
  if (!input || !filter || !output || !input_strides || !filter_strides || !output_strides)
    return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t *is = input_strides, *fs = filter_strides, *os = output_strides;
  return NT_DISPATCH_FLOAT(dtype, [&] {
    using T = scalar_t;
    const nt::tc::ConvProblem prob{input, filter, output, n, c, h, w, k, r, s, pad_h, pad_w, P, Q,
                                   {is[0], is[1], is[2], is[3]}, {fs[0], fs[1], fs[2], fs[3]},
                                   {os[0], os[1], os[2], os[3]}};
    const int rc = nt::tc::try_conv<T>(prob, workspace, workspace_bytes, st);
    if (rc != nt::tc::kNotEligible) return rc;
    nt::simt::Im2col<T> A{static_cast<const T *>(input), c, h, w, r, s, P, Q, pad_h, pad_w,
                          is[0], is[1], is[2], is[3]};
    nt::simt::FilterB<T> B{static_cast<const T *>(filter), r, s, fs[0], fs[1], fs[2], fs[3]};
    nt::simt::StoreConv<T> out{static_cast<T *>(output), P, Q, os[0], os[1], os[2], os[3]};
    return nt::simt::launch_gemm(A, B, out, n * P * Q, k, c * r * s, st);
  });
}

extern "C" int64_t nt_b200_conv2d_workspace_size(int64_t n, int64_t c, int64_t h, int64_t w, int64_t k, int64_t r,
                                                 int64_t s, int64_t pad_h, int64_t pad_w, int dtype) {
  if (n < 0 || c < 0 || h < 0 || w < 0 || k < 0 || r <= 0 || s <= 0 || pad_h < 0 || pad_w < 0) return 0;
  if (!nt::is_half_dtype(dtype)) return 0;
  return nt::tc::conv_workspace_bytes(n, c, h, w, k, r, s, pad_w, 2);
}

// conv2d followed by max_pool2d 3x3 / stride 2 / padding 1 (floor): workspace
// = conv staging, then the conv output (dense NCHW), then the pool counters.
namespace nt {
namespace fused {
inline int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }
struct Plan {
  int64_t P, Q, P2, Q2, staging, y_off, y_bytes, ctr_off, ctr_bytes, total;
};
inline Plan plan(int64_t n, int64_t c, int64_t h, int64_t w, int64_t k, int64_t r, int64_t s, int64_t pad_h,
                 int64_t pad_w) {
  Plan q{};
  q.P = h + 2 * pad_h - r + 1;
  q.Q = w + 2 * pad_w - s + 1;
  q.P2 = q.P > 0 ? (q.P - 1) / 2 + 1 : 0;
  q.Q2 = q.Q > 0 ? (q.Q - 1) / 2 + 1 : 0;
  q.staging = align256(nt::tc::conv_workspace_bytes(n, c, h, w, k, r, s, pad_w, 2));
  q.y_off = q.staging;
  q.y_bytes = align256(n * k * (q.P > 0 ? q.P : 0) * (q.Q > 0 ? q.Q : 0) * 2);
  q.ctr_off = q.y_off + q.y_bytes;
  q.ctr_bytes = n * ((k + 255) / 256) * q.P2 * (int64_t)sizeof(int);
  q.total = q.ctr_off + q.ctr_bytes;
  return q;
}
}  // namespace fused
}  // namespace nt

extern "C" int64_t nt_b200_conv2d_max_pool2d_workspace_size(int64_t n, int64_t c, int64_t h, int64_t w, int64_t k,
                                                            int64_t r, int64_t s, int64_t pad_h, int64_t pad_w,
                                                            int dtype) {
  if (n < 0 || c < 0 || h < 0 || w < 0 || k < 0 || r <= 0 || s <= 0 || pad_h < 0 || pad_w < 0) return 0;
  if (!nt::is_half_dtype(dtype)) return 0;
  return nt::fused::plan(n, c, h, w, k, r, s, pad_h, pad_w).total;
}

extern "C" int nt_b200_conv2d_max_pool2d(const void *input, const void *filter, void *output, int64_t n, int64_t c,
                                         int64_t h, int64_t w, int64_t k, int64_t r, int64_t s, int64_t pad_h,
                                         int64_t pad_w, const int64_t *input_strides, const int64_t *filter_strides,
                                         const int64_t *output_strides, void *workspace, int64_t workspace_bytes,
                                         int pool_in_conv_kernel, int dtype, void *stream) {
  if (n < 0 || c < 0 || h < 0 || w < 0 || k < 0 || r <= 0 || s <= 0 || pad_h < 0 || pad_w < 0 ||
      (pool_in_conv_kernel != 0 && pool_in_conv_kernel != 1))
    return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_half_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  const nt::fused::Plan q = nt::fused::plan(n, c, h, w, k, r, s, pad_h, pad_w);
  if (q.P <= 0 || q.Q <= 0) return NT_B200_ERR_SHAPE_MISMATCH;
  if (n == 0 || k == 0) return 0;
  if (!input || !filter || !output || !input_strides || !filter_strides || !output_strides || !workspace ||
      workspace_bytes < q.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  void *y = ws + q.y_off;
  const int64_t ys[4] = {k * q.P * q.Q, q.P * q.Q, q.Q, 1};
  const int64_t *is = input_strides, *fs = filter_strides, *os = output_strides;
  const int rc = !pool_in_conv_kernel ? nt::tc::kNotEligible : NT_DISPATCH_FLOAT(dtype, [&] {
    using T = scalar_t;
    const nt::tc::ConvProblem prob{input, filter, y, n, c, h, w, k, r, s, pad_h, pad_w, q.P, q.Q,
                                   {is[0], is[1], is[2], is[3]}, {fs[0], fs[1], fs[2], fs[3]},
                                   {ys[0], ys[1], ys[2], ys[3]}};
    const nt::tc::PoolFusion pool{output, {os[0], os[1], os[2], os[3]}, (int)q.P2, (int)q.Q2,
                                  reinterpret_cast<int *>(ws + q.ctr_off)};
    return nt::tc::try_conv<T>(prob, workspace, q.staging, st, &pool);
  });
  if (rc != nt::tc::kNotEligible) return rc;
  // the two kernels: conv2d into the workspace, then max_pool2d (also where
  // the pool does not fit the conv kernel: small images, a narrow row, a
  // layout the tensor-core path does not take)
  const int rc_conv = nt_b200_conv2d(input, filter, y, n, c, h, w, k, r, s, pad_h, pad_w, input_strides,
                                     filter_strides, ys, q.staging > 0 ? workspace : nullptr, q.staging, dtype, stream);
  if (rc_conv != 0) return rc_conv;
  return nt_b200_max_pool2d(y, output, n, k, q.P, q.Q, ys, q.P2, q.Q2, output_strides, 3, 3, 2, 2, 1, 1, dtype,
                            stream);
}

extern "C" int nt_b200_attention(const void *q, const void *k, const void *v, int is_causal, void *o,
                                 int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                                 const int64_t *q_strides, const int64_t *k_strides, const int64_t *v_strides,
                                 const int64_t *o_strides, int dtype, void *stream) {
  if (batch < 0 || heads < 0 || seq_q < 0 || seq_kv < 0 || head_dim < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (head_dim > 128) return NT_B200_ERR_INVALID_ARGUMENT;  // the reference's upper_bound=128 on head_dim
  if (!nt::is_float_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;  // fp32: CUDA-core path
  if (batch * heads * seq_q * head_dim == 0) return 0;
  if (seq_kv == 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !o || !q_strides || !k_strides || !v_strides || !o_strides)
    return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const nt::simt::Strides4 qs{q_strides[0], q_strides[1], q_strides[2], q_strides[3]};
  const nt::simt::Strides4 ks{k_strides[0], k_strides[1], k_strides[2], k_strides[3]};
  const nt::simt::Strides4 vs{v_strides[0], v_strides[1], v_strides[2], v_strides[3]};
  const nt::simt::Strides4 os{o_strides[0], o_strides[1], o_strides[2], o_strides[3]};
  return NT_DISPATCH_FLOAT(dtype, [&] {
    using T = scalar_t;
    // log2(e) rounded to the tensor dtype, as the application's `q * 1.44269504089`
    // rounds the Python constant to q's dtype before multiplying.
    const float log2e_t = static_cast<float>(T(1.44269504089f));
    const nt::tc::AttentionProblem prob{q, k, v, o, batch, heads, seq_q, seq_kv, head_dim, qs.b, qs.h, qs.s, qs.d,
                                        ks.b, ks.h, ks.s, ks.d, vs.b, vs.h, vs.s, vs.d, os.b, os.h, os.s, os.d,
                                        is_causal != 0, log2e_t};
    const int rc = nt::tc::try_attention<T>(prob, st);
    if (rc != nt::tc::kNotEligible) return rc;
    const int64_t rows = batch * heads * seq_q;
    const int64_t grid = (rows + 3) / 4;
    if (grid > (1LL << 31) - 1) return NT_B200_ERR_INVALID_ARGUMENT;
    nt::simt::attention_kernel<T><<<(unsigned)grid, 128, 0, st>>>(
        static_cast<const T *>(q), static_cast<const T *>(k), static_cast<const T *>(v), static_cast<T *>(o), batch,
        heads, seq_q, seq_kv, head_dim, qs, ks, vs, os, is_causal != 0, log2e_t);
    return nt::launch_status();
  });
}
