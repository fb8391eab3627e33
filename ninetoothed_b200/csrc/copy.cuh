// Layout programs: pure data movement, bit for bit, any element type (moved
// as 1-, 2-, 4-, 8- or 16-byte words).
//   clone       tests/test_clone.py:10-47      output[i, j] = input[i, j], any strides
//   to_padded   tests/test_jagged.py:12-49     jagged [B, (len_b), D] -> dense [B, L, D]
//   expand      tests/test_jagged.py:104-143   jagged dst[b, i, :] = src[b, 0, :]
// All three are HBM-bound: each element is read once and written once.
#pragma once

#include <cstring>

#include "common.cuh"

namespace nt {
namespace copy {

// Fixed-size word of W bytes.
template <int W> struct Word;
template <> struct Word<1> { using type = uint8_t; };
template <> struct Word<2> { using type = uint16_t; };
template <> struct Word<4> { using type = uint32_t; };
template <> struct Word<8> { using type = uint2; };
template <> struct Word<16> { using type = uint4; };

// Rows whose columns are contiguous on both sides: each row is `units` words;
// blocks x walk the words of a row, blocks y the rows.
template <typename U>
__global__ void __launch_bounds__(256) rows_kernel(const U *__restrict__ in, U *__restrict__ out, int64_t rows,
                                                   int64_t units, int64_t in_row, int64_t out_row) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const U *src = in + r * in_row;
    U *dst = out + r * out_row;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x)
      dst[u] = src[u];
  }
}

// Any strides: 32 x 32 tiles through shared memory, read along the input's
// faster dimension and written along the output's (element-sized words).
template <typename E>
__global__ void __launch_bounds__(256) tiled_kernel(const E *__restrict__ in, E *__restrict__ out, int64_t rows,
                                                    int64_t cols, int64_t isr, int64_t isc, int64_t osr,
                                                    int64_t osc, bool in_cols_fast, bool out_cols_fast) {
  __shared__ E tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int64_t rb = blockIdx.y; rb * 32 < rows; rb += gridDim.y) {
    const int64_t r0 = rb * 32, c0 = (int64_t)blockIdx.x * 32;
    for (int k = ty; k < 32; k += 8) {
      const int rr = in_cols_fast ? k : tx, cc = in_cols_fast ? tx : k;
      const int64_t r = r0 + rr, c = c0 + cc;
      if (r < rows && c < cols) tile[rr][cc] = in[r * isr + c * isc];
    }
    __syncthreads();
    for (int k = ty; k < 32; k += 8) {
      const int rr = out_cols_fast ? k : tx, cc = out_cols_fast ? tx : k;
      const int64_t r = r0 + rr, c = c0 + cc;
      if (r < rows && c < cols) out[r * osr + c * osc] = tile[rr][cc];
    }
    __syncthreads();
  }
}

// Transpose of 16-bit elements: out[c * out_pitch + r] = in[r * in_pitch + c]
// (the input contiguous along c, the output along r).  A 64 x 64 tile per CTA
// iteration: a thread loads 8 columns of two adjacent rows with two 16-byte
// loads, interleaves them into 8 words of (row 2k, row 2k + 1) pairs in a
// [column][row pair] tile of 32-bit words, then 8 lanes store a column's 64
// rows as one 128-byte run.  The tile's 16-byte chunks are XOR-swizzled by
// column / 8, so both passes are free of bank conflicts.  Tile edges move
// element by element.
__global__ void __launch_bounds__(256) transpose16_kernel(const uint16_t *__restrict__ in, uint16_t *__restrict__ out,
                                                          int64_t rows, int64_t cols, int64_t in_pitch,
                                                          int64_t out_pitch) {
  __shared__ __align__(16) uint32_t tile[64][32];  // [column][row pair]
  const int t = threadIdx.x;
  const int64_t tiles_c = (cols + 63) / 64;
  for (int64_t tb = blockIdx.x; tb < tiles_c * ((rows + 63) / 64); tb += gridDim.x) {
    const int64_t r0 = (tb / tiles_c) * 64, c0 = (tb % tiles_c) * 64;
    {
      const int rp = t / 8, pv = t % 8;  // row pair 0..31, column group 0..7
      const int64_t r = r0 + 2 * rp, c = c0 + 8 * pv;
      uint32_t wa[4] = {0, 0, 0, 0}, wb[4] = {0, 0, 0, 0};
      if (c + 8 <= cols && r + 1 < rows) {
        const uint4 a = __ldcs(reinterpret_cast<const uint4 *>(in + r * in_pitch + c));
        const uint4 b = __ldcs(reinterpret_cast<const uint4 *>(in + (r + 1) * in_pitch + c));
        wa[0] = a.x; wa[1] = a.y; wa[2] = a.z; wa[3] = a.w;
        wb[0] = b.x; wb[1] = b.y; wb[2] = b.z; wb[3] = b.w;
      } else {
        uint16_t ea[8] = {}, eb[8] = {};
        for (int e = 0; e < 8; ++e) {
          if (c + e < cols && r < rows) ea[e] = in[r * in_pitch + c + e];
          if (c + e < cols && r + 1 < rows) eb[e] = in[(r + 1) * in_pitch + c + e];
        }
        for (int j = 0; j < 4; ++j) {
          wa[j] = (uint32_t)ea[2 * j] | ((uint32_t)ea[2 * j + 1] << 16);
          wb[j] = (uint32_t)eb[2 * j] | ((uint32_t)eb[2 * j + 1] << 16);
        }
      }
      const int word = ((rp / 4) ^ pv) * 4 + rp % 4;  // columns pv * 8 + e all have column / 8 == pv
#pragma unroll
      for (int j = 0; j < 4; ++j) {  // word j of a load holds columns 2j (low half) and 2j + 1
        tile[pv * 8 + 2 * j][word] = __byte_perm(wa[j], wb[j], 0x5410);
        tile[pv * 8 + 2 * j + 1][word] = __byte_perm(wa[j], wb[j], 0x7632);
      }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int v = t + 256 * i;
      const int pp = v / 8, cv = v % 8;  // column 0..63, vector of 8 rows 0..7
      const int64_t c = c0 + pp, r = r0 + 8 * cv;
      if (c < cols) {
        const uint4 val = *reinterpret_cast<const uint4 *>(&tile[pp][((cv ^ (pp / 8)) & 7) * 4]);
        if (r + 8 <= rows) {
          __stcs(reinterpret_cast<uint4 *>(out + c * out_pitch + r), val);
        } else {
          const uint16_t *e = reinterpret_cast<const uint16_t *>(&val);
          for (int k = 0; k < 8 && r + k < rows; ++k) out[c * out_pitch + r + k] = e[k];
        }
      }
    }
    __syncthreads();
  }
}

// Transpose of 32-bit elements, same contract as transpose16_kernel: a 32 x 32
// tile per CTA iteration, one 16-byte load of 4 columns and one 16-byte store
// of 4 rows per thread, through a [column][row] tile padded by one word per
// column so that both passes spread over the banks.
__global__ void __launch_bounds__(256) transpose32_kernel(const uint32_t *__restrict__ in, uint32_t *__restrict__ out,
                                                          int64_t rows, int64_t cols, int64_t in_pitch,
                                                          int64_t out_pitch) {
  __shared__ uint32_t tile[32][33];  // [column][row]
  const int t = threadIdx.x;
  const int64_t tiles_c = (cols + 31) / 32;
  for (int64_t tb = blockIdx.x; tb < tiles_c * ((rows + 31) / 32); tb += gridDim.x) {
    const int64_t r0 = (tb / tiles_c) * 32, c0 = (tb % tiles_c) * 32;
    {
      const int rr = t / 8, cv = t % 8;  // row 0..31, group of 4 columns 0..7
      const int64_t r = r0 + rr, c = c0 + 4 * cv;
      uint32_t w[4] = {0, 0, 0, 0};
      if (r < rows && c + 4 <= cols) {
        const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(in + r * in_pitch + c));
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
      } else if (r < rows) {
        for (int e = 0; e < 4; ++e)
          if (c + e < cols) w[e] = in[r * in_pitch + c + e];
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) tile[4 * cv + e][rr] = w[e];
    }
    __syncthreads();
    {
      const int cc = t / 8, rv = t % 8;  // column 0..31, group of 4 rows 0..7
      const int64_t c = c0 + cc, r = r0 + 4 * rv;
      if (c < cols) {
        const uint4 v = make_uint4(tile[cc][4 * rv], tile[cc][4 * rv + 1], tile[cc][4 * rv + 2], tile[cc][4 * rv + 3]);
        if (r + 4 <= rows) {
          __stcs(reinterpret_cast<uint4 *>(out + c * out_pitch + r), v);
        } else {
          const uint32_t e4[4] = {v.x, v.y, v.z, v.w};
          for (int k = 0; k < 4 && r + k < rows; ++k) out[c * out_pitch + r + k] = e4[k];
        }
      }
    }
    __syncthreads();
  }
}

inline int64_t abs64(int64_t v) { return v < 0 ? -v : v; }

template <int W>
int launch_rows(const void *in, void *out, int64_t rows, int64_t row_bytes, int64_t in_row_bytes,
                int64_t out_row_bytes, cudaStream_t stream) {
  using U = typename Word<W>::type;
  const int64_t units = row_bytes / W;
  const unsigned gx = (unsigned)((units + 255) / 256 < 1024 ? (units + 255) / 256 : 1024);
  const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
  rows_kernel<U><<<dim3(gx, gy), 256, 0, stream>>>(static_cast<const U *>(in), static_cast<U *>(out), rows, units,
                                                    in_row_bytes / W, out_row_bytes / W);
  return launch_status();
}

template <typename E>
int launch_tiled(const void *in, void *out, int64_t rows, int64_t cols, int64_t isr, int64_t isc, int64_t osr,
                 int64_t osc, cudaStream_t stream) {
  const bool in_cols_fast = abs64(isc) <= abs64(isr), out_cols_fast = abs64(osc) <= abs64(osr);
  const dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32 < 65535 ? (rows + 31) / 32 : 65535));
  tiled_kernel<E><<<grid, 256, 0, stream>>>(static_cast<const E *>(in), static_cast<E *>(out), rows, cols, isr, isc,
                                            osr, osc, in_cols_fast, out_cols_fast);
  return launch_status();
}

// 2-D copy of `es`-byte elements; strides in elements.
inline int copy2d(const void *in, void *out, int64_t rows, int64_t cols, int64_t isr, int64_t isc, int64_t osr,
                  int64_t osc, int es, cudaStream_t stream) {
  if (rows == 1) isr = osr = 0;  // a single row: only the column strides matter
  if (isc == 1 && osc == 1) {
    // the widest word that divides both base addresses, both row pitches and the row
    const uint64_t bits = reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out) |
                          (uint64_t)(cols * es) | (uint64_t)(abs64(isr) * es) | (uint64_t)(abs64(osr) * es);
    const int64_t row = cols * es, ir = isr * es, orow = osr * es;
    if ((bits & 15u) == 0) return launch_rows<16>(in, out, rows, row, ir, orow, stream);
    if ((bits & 7u) == 0) return launch_rows<8>(in, out, rows, row, ir, orow, stream);
    if ((bits & 3u) == 0) return launch_rows<4>(in, out, rows, row, ir, orow, stream);
    if ((bits & 1u) == 0) return launch_rows<2>(in, out, rows, row, ir, orow, stream);
    return launch_rows<1>(in, out, rows, row, ir, orow, stream);
  }
  if (es == 2 && (reinterpret_cast<uintptr_t>(in) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    // a transpose of 16-bit elements: the input contiguous along one
    // dimension, the output along the other, pitches of whole 16-byte units
    const bool in_c_out_r = isc == 1 && osr == 1 && isr > 0 && osc > 0 && isr % 8 == 0 && osc % 8 == 0;
    const bool in_r_out_c = isr == 1 && osc == 1 && isc > 0 && osr > 0 && isc % 8 == 0 && osr % 8 == 0;
    if (in_c_out_r || in_r_out_c) {
      // out[c * out_pitch + r] = in[r * in_pitch + c] with (rows, cols) swapped for the second case
      const int64_t tr = in_c_out_r ? rows : cols, tc = in_c_out_r ? cols : rows;
      const int64_t tiles = ((tr + 63) / 64) * ((tc + 63) / 64);
      const int64_t cap = (int64_t)sm_count() * 8;
      transpose16_kernel<<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, stream>>>(
          static_cast<const uint16_t *>(in), static_cast<uint16_t *>(out), tr, tc, in_c_out_r ? isr : isc,
          in_c_out_r ? osc : osr);
      return launch_status();
    }
  }
  if (es == 4 && (reinterpret_cast<uintptr_t>(in) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    // the same for 32-bit elements, pitches of whole 16-byte units
    const bool in_c_out_r = isc == 1 && osr == 1 && isr > 0 && osc > 0 && isr % 4 == 0 && osc % 4 == 0;
    const bool in_r_out_c = isr == 1 && osc == 1 && isc > 0 && osr > 0 && isc % 4 == 0 && osr % 4 == 0;
    if (in_c_out_r || in_r_out_c) {
      const int64_t tr = in_c_out_r ? rows : cols, tc = in_c_out_r ? cols : rows;
      const int64_t tiles = ((tr + 31) / 32) * ((tc + 31) / 32);
      const int64_t cap = (int64_t)sm_count() * 8;
      transpose32_kernel<<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, stream>>>(
          static_cast<const uint32_t *>(in), static_cast<uint32_t *>(out), tr, tc, in_c_out_r ? isr : isc,
          in_c_out_r ? osc : osr);
      return launch_status();
    }
  }
  if ((cols + 31) / 32 > 0x7fffffffLL) return NT_B200_ERR_INVALID_ARGUMENT;
  switch (es) {
    case 1: return launch_tiled<uint8_t>(in, out, rows, cols, isr, isc, osr, osc, stream);
    case 2: return launch_tiled<uint16_t>(in, out, rows, cols, isr, isc, osr, osc, stream);
    case 4: return launch_tiled<uint32_t>(in, out, rows, cols, isr, isc, osr, osc, stream);
    default: return launch_tiled<uint2>(in, out, rows, cols, isr, isc, osr, osc, stream);
  }
}

// to_padded: output line (b, i) of `inner` elements = values line
// offsets[b] + i when i < len_b, else `pad` (the padding value's bits).  A
// line is the elements of one ragged position: vs0 / os1 step along the
// ragged dimension, vs1 / os2 along the dense one, whichever tensor
// dimensions those are.
template <typename E>
__global__ void __launch_bounds__(256)
to_padded_kernel(const E *__restrict__ values, const int64_t *__restrict__ offsets, int64_t batch, int64_t max_len,
                 int64_t inner, int64_t vs0, int64_t vs1, E pad, E *__restrict__ out, int64_t os0, int64_t os1,
                 int64_t os2) {
  for (int64_t line = blockIdx.x; line < batch * max_len; line += gridDim.x) {
    const int64_t b = line / max_len, i = line % max_len;
    const int64_t start = offsets[b], len = offsets[b + 1] - start;
    E *dst = out + b * os0 + i * os1;
    if (i < len) {
      const E *src = values + (start + i) * vs0;
      for (int64_t d = threadIdx.x; d < inner; d += blockDim.x) dst[d * os2] = src[d * vs1];
    } else {
      for (int64_t d = threadIdx.x; d < inner; d += blockDim.x) dst[d * os2] = pad;
    }
  }
}

// expand: every line (ragged position) of batch b of the jagged values =
// src[b, :] along the dense dimension.  Block y = batch b; blocks x walk that
// batch's lines.
template <typename E>
__global__ void __launch_bounds__(256)
jagged_expand_kernel(E *__restrict__ values, const int64_t *__restrict__ offsets, int64_t inner, int64_t vs0,
                     int64_t vs1, const E *__restrict__ src, int64_t ss0, int64_t ss2) {
  const int64_t b = blockIdx.y;
  const int64_t start = offsets[b], end = offsets[b + 1];
  const E *s = src + b * ss0;
  for (int64_t line = start + blockIdx.x; line < end; line += gridDim.x) {
    E *dst = values + line * vs0;
    for (int64_t d = threadIdx.x; d < inner; d += blockDim.x) dst[d * vs1] = s[d * ss2];
  }
}

// Element size of a dtype code (0 if unknown).
inline int element_size(int dtype) {
  switch (dtype) {
    case NT_B200_INT8: case NT_B200_UINT8: case NT_B200_FLOAT8_E4M3FN: case NT_B200_FLOAT8_E5M2: return 1;
    case NT_B200_INT16: case NT_B200_UINT16: case NT_B200_FLOAT16: case NT_B200_BFLOAT16: return 2;
    case NT_B200_INT32: case NT_B200_UINT32: case NT_B200_FLOAT32: return 4;
    case NT_B200_INT64: case NT_B200_UINT64: case NT_B200_FLOAT64: return 8;
    default: return 0;
  }
}

// Bits of `value` in the element type of `dtype` (low bytes of the word).
inline bool padding_bits(double value, int dtype, uint64_t *bits) {
  uint64_t b = 0;
  switch (dtype) {
    case NT_B200_FLOAT16: { const __half h = __double2half(value); memcpy(&b, &h, 2); break; }
    case NT_B200_BFLOAT16: { const __nv_bfloat16 h = __double2bfloat16(value); memcpy(&b, &h, 2); break; }
    case NT_B200_FLOAT32: { const float f = (float)value; memcpy(&b, &f, 4); break; }
    case NT_B200_FLOAT64: memcpy(&b, &value, 8); break;
    case NT_B200_INT8: case NT_B200_INT16: case NT_B200_INT32: case NT_B200_INT64:
      b = (uint64_t)(int64_t)value;
      break;
    case NT_B200_UINT8: case NT_B200_UINT16: case NT_B200_UINT32: case NT_B200_UINT64:
      b = (uint64_t)value;
      break;
    default: return false;  // 8-bit floats: no padding conversion
  }
  *bits = b;
  return true;
}

template <typename E>
void launch_to_padded(const void *values, const int64_t *offsets, int64_t batch, int64_t max_len, int64_t inner,
                      int64_t vs0, int64_t vs1, uint64_t pad_bits, void *out, const int64_t *os,
                      cudaStream_t stream) {
  E pad;
  memcpy(&pad, &pad_bits, sizeof(E));
  const int64_t lines = batch * max_len;
  const unsigned grid = (unsigned)(lines < (1 << 19) ? lines : (1 << 19));
  constexpr int64_t per = 16 / (int64_t)sizeof(E);  // elements per 16-byte word
  const bool words = vs1 == 1 && os[2] == 1 && inner % per == 0 && vs0 % per == 0 && os[0] % per == 0 &&
                     os[1] % per == 0 && (reinterpret_cast<uintptr_t>(values) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  if (words) {
    // the dense dimension is contiguous on both sides: lines move as 16-byte
    // words, padding as the pad element repeated across a word
    uint4 pad_word;
    E rep[per];
    for (int64_t k = 0; k < per; ++k) rep[k] = pad;
    memcpy(&pad_word, rep, 16);
    const int64_t o0 = os[0] / per, o1 = os[1] / per;
    to_padded_kernel<uint4><<<grid, 256, 0, stream>>>(static_cast<const uint4 *>(values), offsets, batch, max_len,
                                                      inner / per, vs0 / per, 1, pad_word,
                                                      static_cast<uint4 *>(out), o0, o1, 1);
    return;
  }
  to_padded_kernel<E><<<grid, 256, 0, stream>>>(static_cast<const E *>(values), offsets, batch, max_len, inner, vs0,
                                                vs1, pad, static_cast<E *>(out), os[0], os[1], os[2]);
}

template <typename E>
void launch_expand(void *values, const int64_t *offsets, int64_t batch, int64_t inner, int64_t vs0, int64_t vs1,
                   const void *src, int64_t ss0, int64_t ss2, cudaStream_t stream) {
  const int64_t per_batch = sm_count() * 8 / batch + 1;
  const dim3 grid((unsigned)(per_batch < 1024 ? per_batch : 1024), (unsigned)batch);
  constexpr int64_t per = 16 / (int64_t)sizeof(E);  // elements per 16-byte word
  if (vs1 == 1 && ss2 == 1 && inner % per == 0 && vs0 % per == 0 && ss0 % per == 0 &&
      (reinterpret_cast<uintptr_t>(values) & 15u) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    // the dense dimension is contiguous on both sides: lines as 16-byte words
    jagged_expand_kernel<uint4><<<grid, 256, 0, stream>>>(static_cast<uint4 *>(values), offsets, inner / per,
                                                          vs0 / per, 1, static_cast<const uint4 *>(src), ss0 / per,
                                                          1);
    return;
  }
  jagged_expand_kernel<E><<<grid, 256, 0, stream>>>(static_cast<E *>(values), offsets, inner, vs0, vs1,
                                                    static_cast<const E *>(src), ss0, ss2);
}

}  // namespace copy
}  // namespace nt

extern "C" int nt_b200_clone(const void *input, void *output, int64_t rows, int64_t cols, int64_t input_stride_row,
                             int64_t input_stride_col, int64_t output_stride_row, int64_t output_stride_col,
                             int dtype, void *stream) {
  const int es = nt::copy::element_size(dtype);
  if (es == 0) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (rows < 0 || cols < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (rows == 0 || cols == 0) return 0;
  if (!input || !output) return NT_B200_ERR_INVALID_ARGUMENT;
  return nt::copy::copy2d(input, output, rows, cols, input_stride_row, input_stride_col, output_stride_row,
                          output_stride_col, es, static_cast<cudaStream_t>(stream));
}

extern "C" int nt_b200_jagged_to_padded(const void *values, const int64_t *offsets, int64_t batch, int64_t inner,
                                        int64_t values_stride_ragged, int64_t values_stride_inner, double padding,
                                        void *output, int64_t max_len, const int64_t *output_strides, int dtype,
                                        void *stream) {
  const int es = nt::copy::element_size(dtype);
  uint64_t pad = 0;
  if (es == 0 || !nt::copy::padding_bits(padding, dtype, &pad)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || inner < 0 || max_len < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (batch == 0 || inner == 0 || max_len == 0) return 0;
  if (!values || !offsets || !output || !output_strides) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t vr = values_stride_ragged, vi = values_stride_inner;
  switch (es) {
    case 1: nt::copy::launch_to_padded<uint8_t>(values, offsets, batch, max_len, inner, vr, vi, pad, output,
                                                output_strides, st); break;
    case 2: nt::copy::launch_to_padded<uint16_t>(values, offsets, batch, max_len, inner, vr, vi, pad, output,
                                                 output_strides, st); break;
    case 4: nt::copy::launch_to_padded<uint32_t>(values, offsets, batch, max_len, inner, vr, vi, pad, output,
                                                 output_strides, st); break;
    default: nt::copy::launch_to_padded<uint64_t>(values, offsets, batch, max_len, inner, vr, vi, pad, output,
                                                  output_strides, st); break;
  }
  return nt::launch_status();
}

extern "C" int nt_b200_jagged_expand(void *values, const int64_t *offsets, int64_t batch, int64_t inner,
                                     int64_t values_stride_ragged, int64_t values_stride_inner, const void *src,
                                     int64_t src_stride_batch, int64_t src_stride_inner, int dtype, void *stream) {
  const int es = nt::copy::element_size(dtype);
  if (es == 0) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || inner < 0 || batch > 65535) return NT_B200_ERR_INVALID_ARGUMENT;
  if (batch == 0 || inner == 0) return 0;
  if (!values || !offsets || !src) return NT_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t vr = values_stride_ragged, vi = values_stride_inner, sb = src_stride_batch, si = src_stride_inner;
  switch (es) {
    case 1: nt::copy::launch_expand<uint8_t>(values, offsets, batch, inner, vr, vi, src, sb, si, st); break;
    case 2: nt::copy::launch_expand<uint16_t>(values, offsets, batch, inner, vr, vi, src, sb, si, st); break;
    case 4: nt::copy::launch_expand<uint32_t>(values, offsets, batch, inner, vr, vi, src, sb, si, st); break;
    default: nt::copy::launch_expand<uint64_t>(values, offsets, batch, inner, vr, vi, src, sb, si, st); break;
  }
  return nt::launch_status();
}
