/*
 * nt_b200.h -- C ABI of the B200 (sm_100a) kernel library `libnt_b200.so`.
 *
 * One entry point per operator family that NineToothed's arrange-and-apply
 * programs generate.  Every entry point:
 *   - takes raw device pointers, int64 sizes and element strides, a dtype code
 *     and the caller's CUDA stream (a `cudaStream_t` passed as `void*`);
 *   - never allocates device memory and never synchronises the stream;
 *   - returns 0 on success, a `cudaError_t` value when a launch fails, or one of
 *     the NT_B200_ERR_* codes below when the arguments are rejected on the host
 *     before anything is launched;
 *   - launches nothing when an output has zero elements (returns 0), the same
 *     empty-launch rule as the reference runtime (src/ninetoothed/compiler/
 *     runtime.py:1411-1422).
 *
 * The shape of this ABI follows the launcher the reference CUDA backend emits
 * (src/ninetoothed/backends/emitters/cuda.py:368-380: `extern "C" int
 * launch_<kernel>(..., cudaStream_t stream)` returning `cudaGetLastError()`),
 * with the per-tensor pointer/shape/stride triples that the reference runtime
 * binds (src/ninetoothed/compiler/runtime.py:1301-1332).  Dtype codes are the
 * values of the reference's `NineToothedDataType` enum
 * (src/ninetoothed/backends/materializers/cpp.py:10-23, 26-58).
 */
#ifndef NT_B200_H
#define NT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types: the NineToothedDataType values of the reference ABI (0-11),
 * extended with the two 8-bit float types the reference's matmul/addmm tests
 * use (torch.float8_e4m3fn, torch.float8_e5m2), which its C++ ABI enum lacks. */
enum NtB200DataType {
    NT_B200_INT8 = 0,
    NT_B200_INT16 = 1,
    NT_B200_INT32 = 2,
    NT_B200_INT64 = 3,
    NT_B200_UINT8 = 4,
    NT_B200_UINT16 = 5,
    NT_B200_UINT32 = 6,
    NT_B200_UINT64 = 7,
    NT_B200_FLOAT16 = 8,
    NT_B200_BFLOAT16 = 9,
    NT_B200_FLOAT32 = 10,
    NT_B200_FLOAT64 = 11,
    NT_B200_FLOAT8_E4M3FN = 12,
    NT_B200_FLOAT8_E5M2 = 13
};

/* Host-side argument errors (no launch happened).  Values are above the
 * cudaError_t range used by CUDA 12 so the two never collide. */
#define NT_B200_ERR_INVALID_ARGUMENT 10001 /* null pointer, negative size, bad window */
#define NT_B200_ERR_UNSUPPORTED_DTYPE 10002 /* dtype not implemented for this op */
#define NT_B200_ERR_SHAPE_MISMATCH 10003   /* output shape inconsistent with inputs */
#define NT_B200_ERR_NO_DEVICE 10004        /* no sm_100 device current */
#define NT_B200_ERR_DEVICE_TIMEOUT 10005   /* a bounded device-side wait gave up */
#define NT_B200_ERR_WORKSPACE_TOO_LARGE 10006 /* staging exceeds the library's fixed array */

/* Library identity and diagnostics. */
int nt_b200_version(void);
const char *nt_b200_error_string(int code);

/*
 * Reads and clears the device-side error word of the current device after
 * synchronising `stream`.  Pipelined kernels (GEMM, attention, conv) bound every
 * mbarrier wait; a wait that runs out records NT_B200_ERR_DEVICE_TIMEOUT there
 * and the kernel returns early instead of hanging.  `*status` receives 0 or that
 * code.  No counterpart in the reference (its launchers only report launch
 * errors, src/ninetoothed/compiler/runtime.py:31-35).
 */
int nt_b200_device_status(void *stream, int *status);

/*
 * Row softmax over the last dimension: y = exp(x - max(x)) / sum(exp(x - max(x))),
 * fp32 internal math, result rounded to `dtype`.  Replaces the launcher of
 * `softmax_kernel` (tests/test_softmax.py:10-27 in the reference; one program per
 * row, `BLOCK_SIZE = cols`).  dtype: FLOAT16, BFLOAT16, FLOAT32.
 */
int nt_b200_softmax(const void *input, void *output, int64_t rows, int64_t cols,
                    int64_t input_stride_row, int64_t input_stride_col,
                    int64_t output_stride_row, int64_t output_stride_col,
                    int dtype, void *stream);

/*
 * output[i] = lhs[i] + rhs[i] for i < size.  Replaces `add_kernel`
 * (tests/test_add.py:9-24).  dtype: FLOAT16, BFLOAT16, FLOAT32.
 */
int nt_b200_add(const void *lhs, const void *rhs, void *output, int64_t size,
                int64_t lhs_stride, int64_t rhs_stride, int64_t output_stride,
                int dtype, void *stream);

/*
 * output[i] = pow(input[i], exponent[i]) (CUDA powf, fp32 math).  Replaces
 * `pow_kernel` (tests/test_pow.py:10-31, `libdevice.pow`).
 * dtype: FLOAT16, BFLOAT16, FLOAT32.
 */
int nt_b200_pow(const void *input, const void *exponent, void *output, int64_t size,
                int64_t input_stride, int64_t exponent_stride,
                int64_t output_stride, int dtype, void *stream);

/*
 * output[i] = rand(seed, i) > p ? input[i] / (1 - p) : 0, where rand is
 * Philox4x32-10 on counter (i, 0, 0, 0) with key (seed lo, seed hi), first word
 * mapped to [0, 1) as Triton's `tl.rand` does.  Replaces `dropout_kernel`
 * (tests/test_dropout.py:12-29).  dtype: FLOAT16, BFLOAT16, FLOAT32.
 */
int nt_b200_dropout(const void *input, float p, int64_t seed, void *output,
                    int64_t size, int64_t input_stride, int64_t output_stride,
                    int dtype, void *stream);

/*
 * 2-D max pooling over NCHW tensors: output[n,c,p,q] = max over the window rows
 * p*stride_h - pad_h + [0, window_h) and columns q*stride_w - pad_w + [0,
 * window_w) of input, skipping positions outside the input (the reference's
 * `other=-inf` fill).  `out_h`/`out_w` are the caller's output extents (floor or
 * ceil mode is decided by the caller, as in tests/test_max_pool2d.py:39-61).
 * Bit-exact.  Strides are element strides of the 4-D tensors.
 * dtype: FLOAT16, BFLOAT16, FLOAT32.
 */
int nt_b200_max_pool2d(const void *input, void *output, int64_t n, int64_t c,
                       int64_t h, int64_t w, const int64_t *input_strides,
                       int64_t out_h, int64_t out_w, const int64_t *output_strides,
                       int64_t window_h, int64_t window_w, int64_t stride_h,
                       int64_t stride_w, int64_t pad_h, int64_t pad_w, int dtype,
                       void *stream);

/*
 * output[M,N] = cast_out(cast_f16(sum_k lhs[m,k] * rhs[k,n])) with an fp32
 * accumulator: the `matmul` application (tests/test_matmul.py:41-47) rounds the
 * accumulator to float16 before the store converts it to the output dtype.
 * in_dtype: FLOAT16, BFLOAT16, FLOAT8_E4M3FN or FLOAT8_E5M2 (both operands;
 * 8-bit operands run on tcgen05 kind::f8f6f4) or FLOAT32 (exact fp32 on CUDA
 * cores); out_dtype: FLOAT16, BFLOAT16, FLOAT32.  Strides are element strides (row, col) of each 2-D operand.
 */
int nt_b200_matmul(const void *lhs, const void *rhs, void *output, int64_t m,
                   int64_t n, int64_t k, int64_t lhs_stride_row,
                   int64_t lhs_stride_col, int64_t rhs_stride_row,
                   int64_t rhs_stride_col, int64_t output_stride_row,
                   int64_t output_stride_col, int in_dtype, int out_dtype,
                   void *stream);

/*
 * output = beta * input + alpha * cast_f16(mat1 @ mat2), stored in out_dtype:
 * the `addmm` application (tests/test_addmm.py:13-38), whose inlined matmul
 * rounds the fp32 accumulator to float16.  The epilogue follows Triton's typing
 * of a scalar argument against a tensor: beta * input in in_dtype, alpha * the
 * float16 product in float16, their sum in float16 when in_dtype is FLOAT16
 * (fp32 otherwise).  `input` has the output's [M,N] shape and in_dtype.
 */
int nt_b200_addmm(const void *input, const void *mat1, const void *mat2, float beta,
                  float alpha, void *output, int64_t m, int64_t n, int64_t k,
                  int64_t input_stride_row, int64_t input_stride_col,
                  int64_t mat1_stride_row, int64_t mat1_stride_col,
                  int64_t mat2_stride_row, int64_t mat2_stride_col,
                  int64_t output_stride_row, int64_t output_stride_col,
                  int in_dtype, int out_dtype, void *stream);

/*
 * Flash attention with the reference application's numerics
 * (tests/test_attention.py:44-70): q' = round(q * round(log2 e)) in the input
 * dtype, s = q' k^T in fp32 (softmax scale 1; callers pre-scale q), keys beyond
 * seq_kv masked, optional causal mask (query index >= key index), base-2 online
 * softmax with fp32 running max/sum, p rounded to the input dtype before p @ v,
 * o = acc / l.  Tensors are [batch, heads, seq, head_dim]; strides are 4-entry
 * element-stride arrays.  dtype: FLOAT16 or BFLOAT16 (q, k, v and o; tcgen05) or
 * FLOAT32 (CUDA cores).
 */
int nt_b200_attention(const void *q, const void *k, const void *v, int is_causal,
                      void *o, int64_t batch, int64_t heads, int64_t seq_q,
                      int64_t seq_kv, int64_t head_dim, const int64_t *q_strides,
                      const int64_t *k_strides, const int64_t *v_strides,
                      const int64_t *o_strides, int dtype, void *stream);

/*
 * conv2d as an implicit GEMM (tests/test_conv2d.py:14-49 arrangement with the
 * matmul application): output[n,k,p,q] = cast_out(cast_f16(sum over (c,r,s) of
 * input[n,c,p+r-pad_h,q+s-pad_w] * filter[k,c,r,s])), zero outside the input,
 * stride 1, fp32 accumulation.  NCHW input/output, KCRS filter; strides are
 * 4-entry element-stride arrays.  dtype: FLOAT16 or BFLOAT16 (all three tensors).
 *
 * `workspace` is caller-owned device memory of at least
 * nt_b200_conv2d_workspace_size(...) bytes, 256-byte aligned; the tensor-core
 * path stages the input as NHWC and the filter as KRSC there.  With a smaller
 * (or null) workspace the call takes the CUDA-core path instead.
 */
int nt_b200_conv2d(const void *input, const void *filter, void *output, int64_t n,
                   int64_t c, int64_t h, int64_t w, int64_t k, int64_t r, int64_t s,
                   int64_t pad_h, int64_t pad_w, const int64_t *input_strides,
                   const int64_t *filter_strides, const int64_t *output_strides,
                   void *workspace, int64_t workspace_bytes, int dtype, void *stream);

/*
 * conv2d followed by max_pool2d with a 3x3 window, stride 2, padding 1 (floor
 * mode): output[n, k, i, j] = max_pool2d(conv2d(input, filter, padding))[n, k,
 * i, j], bit-identical to the two programs run one after the other
 * (nt_b200_conv2d, then nt_b200_max_pool2d), output [n, k, P2, Q2] with
 * P2 = (P - 1) / 2 + 1, Q2 = (Q - 1) / 2 + 1 for the conv extents P, Q.  The
 * conv result goes to the workspace.  pool_in_conv_kernel = 0 pools it with
 * the max_pool2d kernel after the conv kernel (the faster order on B200);
 * pool_in_conv_kernel = 1 pools inside the tensor-core conv kernel where the
 * shape allows (extra pool warps per CTA read each pool row back from L2 once
 * the warp that completes its last input rows hands it over) and falls back to
 * the two kernels elsewhere.  `workspace` (256-byte aligned) must hold
 * nt_b200_conv2d_max_pool2d_workspace_size(...) bytes (conv staging + the conv
 * result + counters).  No single program of the reference does this; it
 * composes its conv2d and max_pool2d programs (tests/test_conv2d.py,
 * tests/test_max_pool2d.py).
 */
int nt_b200_conv2d_max_pool2d(const void *input, const void *filter, void *output,
                              int64_t n, int64_t c, int64_t h, int64_t w, int64_t k,
                              int64_t r, int64_t s, int64_t pad_h, int64_t pad_w,
                              const int64_t *input_strides, const int64_t *filter_strides,
                              const int64_t *output_strides, void *workspace,
                              int64_t workspace_bytes, int pool_in_conv_kernel, int dtype,
                              void *stream);
int64_t nt_b200_conv2d_max_pool2d_workspace_size(int64_t n, int64_t c, int64_t h, int64_t w,
                                                 int64_t k, int64_t r, int64_t s,
                                                 int64_t pad_h, int64_t pad_w, int dtype);

/*
 * Workspace bytes the tensor-core conv2d path needs for this problem (0 when
 * the path does not apply: 32-bit dtype or channels not a multiple of 8): the
 * input as NHWC with pad_w zero columns on each side of every row, then the
 * filter as KRSC.  No counterpart in the reference (its conv2d program stages
 * nothing).
 */
int64_t nt_b200_conv2d_workspace_size(int64_t n, int64_t c, int64_t h, int64_t w,
                                      int64_t k, int64_t r, int64_t s, int64_t pad_h,
                                      int64_t pad_w, int dtype);

/*
 * conv2d exactly as nt_b200_conv2d, for callers that cannot provide device
 * memory at call time: a C host program without a device allocator, a loop
 * that must not call cudaMalloc (it synchronises the device and stalls other
 * streams), or an application whose memory budget is fixed at start-up.  The
 * NHWC/KRSC staging goes to a 64 MiB array inside the library (held on every
 * GPU that loads the library until the process exits); the call allocates
 * nothing.  Problems needing more staging than 64 MiB return
 * NT_B200_ERR_WORKSPACE_TOO_LARGE without launching.  All calls on a device
 * share the array, so calls whose kernels overlap on the GPU race; calls on
 * one stream are safe.  The first call on a device looks the array's address
 * up with that device current; make it before any stream capture.
 * No counterpart in the reference.
 */
int nt_b200_conv2d_no_alloc(const void *input, const void *filter, void *output,
                            int64_t n, int64_t c, int64_t h, int64_t w, int64_t k,
                            int64_t r, int64_t s, int64_t pad_h, int64_t pad_w,
                            const int64_t *input_strides,
                            const int64_t *filter_strides,
                            const int64_t *output_strides, int dtype, void *stream);

/*
 * clone (tests/test_clone.py:10-47, all four applications): output[i, j] =
 * input[i, j] for a rows x cols matrix with any element strides; a bit copy
 * of any dtype code 0-13.
 */
int nt_b200_clone(const void *input, void *output, int64_t rows, int64_t cols,
                  int64_t input_stride_row, int64_t input_stride_col,
                  int64_t output_stride_row, int64_t output_stride_col, int dtype,
                  void *stream);

/*
 * to_padded_tensor (tests/test_jagged.py:12-49): a jagged 3-D tensor with one
 * ragged dimension -- packed `values` holding element (b, r, d) at
 * (offsets[b] + r) * values_stride_ragged + d * values_stride_inner, device
 * `offsets` [batch + 1] (int64), `inner` elements along the dense dimension --
 * to a dense `output` whose element (b, r, d) sits at output_strides[0] * b +
 * output_strides[1] * r + output_strides[2] * d for r < max_len; positions
 * r >= len_b hold `padding` converted to the dtype (codes 0-11).  Ragged
 * dimension 1: the strides of values [total, D] in order; ragged dimension 2:
 * values [D, total] with its strides swapped.
 */
int nt_b200_jagged_to_padded(const void *values, const int64_t *offsets, int64_t batch,
                             int64_t inner, int64_t values_stride_ragged,
                             int64_t values_stride_inner, double padding, void *output,
                             int64_t max_len, const int64_t *output_strides, int dtype,
                             void *stream);

/*
 * Copy with expand into a jagged tensor (tests/test_jagged.py:104-143): every
 * element (b, r, d) of the jagged tensor (layout as above) becomes
 * src[b * src_stride_batch + d * src_stride_inner], the dense source being
 * broadcast along the ragged dimension.  batch <= 65535.
 */
int nt_b200_jagged_expand(void *values, const int64_t *offsets, int64_t batch, int64_t inner,
                          int64_t values_stride_ragged, int64_t values_stride_inner,
                          const void *src, int64_t src_stride_batch, int64_t src_stride_inner,
                          int dtype, void *stream);

/*
 * Failure-detection self-test (no counterpart in the reference): launches one
 * thread that waits on an mbarrier nothing ever arrives on, through the same
 * bounded wait the pipelined kernels use, with a limit of `limit_ns`
 * (1 us .. 1 s).  The wait gives up, records NT_B200_ERR_DEVICE_TIMEOUT in the
 * device error word and the kernel exits; nt_b200_device_status then reports
 * it.  The context stays usable.
 */
int nt_b200_wait_timeout_selftest(int64_t limit_ns, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NT_B200_H */
