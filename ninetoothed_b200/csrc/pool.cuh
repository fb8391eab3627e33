// 2-D max pooling (the reference's `max_pool2d` arrangement/application,
// tests/test_max_pool2d.py:13-36, and its padded stride-2 variant).
//
// Window positions outside the input are skipped, which is the same as the
// reference's `other=-inf` fill for a max.  The result is an element of the
// input, so it is bit-exact.  Neighbouring windows overlap; the overlap is
// served from L1, so HBM sees each input element about once.
#pragma once

#include "common.cuh"

namespace nt {
namespace pool {

template <typename T>
__global__ void __launch_bounds__(256)
max_pool2d_kernel(const T *__restrict__ in, T *__restrict__ out, int64_t n, int64_t c, int64_t h,
                  int64_t w, int64_t isn, int64_t isc, int64_t ish, int64_t isw, int64_t out_h,
                  int64_t out_w, int64_t osn, int64_t osc, int64_t osh, int64_t osw, int wh, int ww,
                  int sh, int sw, int ph, int pw) {
  const int64_t total = n * c * out_h * out_w;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = idx % out_w;
    int64_t t = idx / out_w;
    const int64_t p = t % out_h;
    t /= out_h;
    const int64_t ci = t % c;
    const int64_t ni = t / c;
    const T *plane = in + ni * isn + ci * isc;
    const int64_t h0 = p * sh - ph, w0 = q * sw - pw;
    float m = -INFINITY;
    for (int r = 0; r < wh; ++r) {
      const int64_t y = h0 + r;
      if (y < 0 || y >= h) continue;
      const T *row = plane + y * ish;
      for (int s = 0; s < ww; ++s) {
        const int64_t x = w0 + s;
        if (x < 0 || x >= w) continue;
        const float v = to_f(row[x * isw]);
        m = v > m ? v : m;
      }
    }
    out[ni * osn + ci * osc + p * osh + q * osw] = from_f<T>(m);
  }
}

// Row path for inputs and outputs with unit column stride: one warp per output
// row (n, c, p), lanes over the output columns, so index arithmetic is per row
// and a warp's loads are one contiguous run of the input row.  WH/WW/SH/SW > 0
// fix the window and stride at compile time (fully unrolled, all window loads
// in flight together); 0 takes them from the arguments.
template <typename T, int WH, int WW, int SH, int SW>
__global__ void __launch_bounds__(256)
max_pool2d_rows_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int H, int W, int P, int Q,
                       int64_t isn, int64_t isc, int64_t ish, int64_t osn, int64_t osc, int64_t osp, int64_t rows,
                       int wh_, int ww_, int sh_, int sw_, int ph, int pw) {
  const int wh = WH > 0 ? WH : wh_, ww = WW > 0 ? WW : ww_;
  const int sh = SH > 0 ? SH : sh_, sw = SW > 0 ? SW : sw_;
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += (int64_t)gridDim.x * 8) {
    const int p = (int)(row % P);
    const int64_t nc = row / P;
    const int ci = (int)(nc % C);
    const int64_t ni = nc / C;
    const T *plane = in + ni * isn + ci * isc;
    T *orow = out + ni * osn + ci * osc + p * osp;
    const int y0 = p * sh - ph;
    for (int q = lane; q < Q; q += 32) {
      const int x0 = q * sw - pw;
      float m = -INFINITY;
#pragma unroll
      for (int r = 0; r < (WH > 0 ? WH : 1); ++r) {
        for (int rr = (WH > 0 ? r : 0); rr < (WH > 0 ? r + 1 : wh); ++rr) {
          const int y = y0 + rr;
          if (y < 0 || y >= H) continue;
          const T *irow = plane + y * ish;
#pragma unroll
          for (int s2 = 0; s2 < (WW > 0 ? WW : 1); ++s2) {
            for (int ss = (WW > 0 ? s2 : 0); ss < (WW > 0 ? s2 + 1 : ww); ++ss) {
              const int x = x0 + ss;
              if (x < 0 || x >= W) continue;
              const float v = to_f(irow[x]);
              m = v > m ? v : m;
            }
          }
        }
      }
      orow[q] = from_f<T>(m);
    }
  }
}

// Fixed-window row-pair path: each lane computes output column q of two
// consecutive output rows.  All (SH + WH) x WW window loads of the pair are
// issued up front from clamped (always valid) addresses and the out-of-image
// ones are replaced by -inf afterwards, so a warp keeps every load in flight at
// once instead of waiting on them one by one.
// Grid: x = plane (n, c), y = chunk of 8 row pairs (one per warp), so the
// only division is one 32-bit n/c split per warp.
template <typename T, int WH, int WW, int SH, int SW>
__global__ void __launch_bounds__(256)
max_pool2d_pairs_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int H, int W, int P, int Q,
                        int64_t isn, int64_t isc, int64_t ish, int64_t osn, int64_t osc, int64_t osp, int ph,
                        int pw) {
  constexpr int NR = SH + WH;  // input rows feeding two output rows
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (pair * 2 < P) {
    const int p = pair * 2;
    const unsigned plane_idx = blockIdx.x;
    const int ci = (int)(plane_idx % (unsigned)C);
    const int64_t ni = plane_idx / (unsigned)C;
    const T *plane = in + ni * isn + ci * isc;
    T *orow = out + ni * osn + ci * osc + p * osp;
    const int y0 = p * SH - ph;
    const bool second = p + 1 < P;
    for (int q = lane; q < Q; q += 32) {
      const int x0 = q * SW - pw;
      float v[NR][WW];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const int y = y0 + r;
        const int yc = min(max(y, 0), H - 1);
        const T *irow = plane + (int64_t)yc * ish;
#pragma unroll
        for (int s2 = 0; s2 < WW; ++s2) {
          const int xc = min(max(x0 + s2, 0), W - 1);
          v[r][s2] = to_f(irow[xc]);
        }
      }
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const bool y_ok = (unsigned)(y0 + r) < (unsigned)H;
#pragma unroll
        for (int s2 = 0; s2 < WW; ++s2) {
          const bool ok = y_ok && (unsigned)(x0 + s2) < (unsigned)W;
          v[r][s2] = ok ? v[r][s2] : -INFINITY;
        }
      }
      float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
      for (int r = 0; r < WH; ++r)
#pragma unroll
        for (int s2 = 0; s2 < WW; ++s2) {
          m0 = v[r][s2] > m0 ? v[r][s2] : m0;
          m1 = v[r + SH][s2] > m1 ? v[r + SH][s2] : m1;
        }
      orow[q] = from_f<T>(m0);
      if (second) orow[osp + q] = from_f<T>(m1);
    }
  }
}

// 3x3 window, stride 2, padding 1 (the pooling that follows conv2d in the
// benchmark configuration), 16- or 32-bit elements, even row length, rows
// starting on a pair boundary.  Lane q
// loads the element pair (2q, 2q+1) of each input row as one vector and the
// element 2q-1 as a scalar (an L1 hit: the neighbouring lane's pair), takes the
// horizontal 3-max in the element type, and the vertical maxima over the 5
// input rows shared by output rows p and p+1.  The max of elements is exact,
// so no conversion is needed.
template <typename T> struct Pair;
template <> struct Pair<__half> { using V = __half2; };
template <> struct Pair<__nv_bfloat16> { using V = __nv_bfloat162; };
template <> struct Pair<float> { using V = float2; };

__device__ __forceinline__ __half vmax(__half a, __half b) { return __hmax(a, b); }
__device__ __forceinline__ __nv_bfloat16 vmax(__nv_bfloat16 a, __nv_bfloat16 b) { return __hmax(a, b); }
__device__ __forceinline__ float vmax(float a, float b) { return fmaxf(a, b); }
template <typename T> __device__ __forceinline__ T neg_inf() { return from_f<T>(-INFINITY); }

template <typename T>
__global__ void __launch_bounds__(256)
max_pool2d_3x3s2p1_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int H, int W, int P, int Q,
                          int64_t isn, int64_t isc, int64_t ish, int64_t osn, int64_t osc, int64_t osp) {
  using V = typename Pair<T>::V;
  constexpr int PAIRS = 2;  // row pairs per warp, loaded together
  const int lane = threadIdx.x & 31;
  const int first_pair = (blockIdx.y * 8 + (threadIdx.x >> 5)) * PAIRS;
  if (first_pair * 2 >= P) return;
  const unsigned plane_idx = blockIdx.x;
  const int ci = (int)(plane_idx % (unsigned)C);
  const int64_t ni = plane_idx / (unsigned)C;
  const T *plane = in + ni * isn + ci * isc;
  T *oplane = out + ni * osn + ci * osc;
  const T ninf = neg_inf<T>();
  for (int q = lane; q < Q; q += 32) {
    const int x = 2 * q;  // window columns x-1, x, x+1
    const bool pair_ok = x < W;  // W is even, so x + 1 < W too
    T hm[PAIRS][5];
#pragma unroll
    for (int u = 0; u < PAIRS; ++u) {
      const int y0 = 4 * (first_pair + u) - 1;  // output rows p = 2 * pair, p + 1
#pragma unroll
      for (int r = 0; r < 5; ++r) {
        const int y = y0 + r;
        const bool y_ok = (unsigned)y < (unsigned)H;
        const T *irow = plane + (int64_t)(y_ok ? y : 0) * ish;
        const V v = *reinterpret_cast<const V *>(irow + (pair_ok ? x : 0));
        const T left = irow[x > 0 ? x - 1 : 0];
        // x <= W always (the ABI rejects windows that start past the padded
        // input), so column x - 1 is inside the row whenever x > 0.
        T m = pair_ok ? vmax(reinterpret_cast<const T *>(&v)[0], reinterpret_cast<const T *>(&v)[1]) : ninf;
        m = x > 0 ? vmax(m, left) : m;
        hm[u][r] = y_ok ? m : ninf;
      }
    }
#pragma unroll
    for (int u = 0; u < PAIRS; ++u) {
      const int p = 2 * (first_pair + u);
      if (p < P) oplane[(int64_t)p * osp + q] = vmax(vmax(hm[u][0], hm[u][1]), hm[u][2]);
      if (p + 1 < P) oplane[(int64_t)(p + 1) * osp + q] = vmax(vmax(hm[u][2], hm[u][3]), hm[u][4]);
    }
  }
}

// Vector form of the 3x3 / stride 2 / padding 1 path for 16-bit elements, row
// length W <= 64 with W % 8 == 0 and Q % 4 == 0 (56 -> 28 in the benchmark
// config).  An 8-lane group owns one pair of output rows: lane j loads input
// columns [8j, 8j + 8) of each of the 5 input rows with one 16-byte load,
// takes column 8j - 1 from lane j - 1 by a shuffle, and writes output
// columns [4j, 4j + 4) of both rows with 8-byte stores.  A warp covers 4 row
// pairs, so 20 16-byte loads per lane group are in flight together.
template <typename T>
__global__ void __launch_bounds__(256)
max_pool2d_3x3s2p1_vec_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int H, int W, int P, int Q,
                              int64_t isn, int64_t isc, int64_t ish, int64_t osn, int64_t osc, int64_t osp,
                              int pairs_per_plane, int64_t total_pairs) {
  // launched as a programmatic dependent (launch_overlapped); no early
  // trigger for the next kernel: this grid runs several waves, and dependents
  // let in from its last wave on made it slower
  wait_prior_grid();
  const int lane = threadIdx.x & 31;
  const int j = lane & 7;  // lane within the group
  const int64_t g = (int64_t)blockIdx.x * 32 + (threadIdx.x >> 3);
  const bool active = g < total_pairs;
  const int64_t gg = active ? g : 0;
  const unsigned plane_idx = (unsigned)(gg / pairs_per_plane);
  const int pair = (int)(gg - (int64_t)plane_idx * pairs_per_plane);
  const int ci = (int)(plane_idx % (unsigned)C);
  const int64_t ni = plane_idx / (unsigned)C;
  const T *plane = in + ni * isn + ci * isc;
  const int p = 2 * pair;
  const int y0 = 2 * p - 1;
  const bool col_ok = 8 * j < W;
  const T ninf = neg_inf<T>();
  T hm[5][4];
#pragma unroll
  for (int r = 0; r < 5; ++r) {
    const int y = y0 + r;
    const bool y_ok = (unsigned)y < (unsigned)H;
    const T *irow = plane + (int64_t)(y_ok ? y : 0) * ish;
    int4 raw = make_int4(0, 0, 0, 0);
    if (active && col_ok) raw = *reinterpret_cast<const int4 *>(irow + 8 * j);
    const T *x = reinterpret_cast<const T *>(&raw);
    // column 8j - 1 is the last element held by lane j - 1 (padding for j = 0)
    const unsigned short last = reinterpret_cast<const unsigned short *>(&raw)[7];
    const unsigned short prev_bits = (unsigned short)__shfl_up_sync(0xffffffffu, (unsigned)last, 1, 8);
    T left;
    *reinterpret_cast<unsigned short *>(&left) = prev_bits;
    if (j == 0) left = ninf;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const T l = k == 0 ? left : x[2 * k - 1];
      const T m = vmax(vmax(l, x[2 * k]), x[2 * k + 1]);
      hm[r][k] = (y_ok && col_ok) ? m : ninf;
    }
  }
  if (!active || 4 * j >= Q) return;
  T *orow = out + ni * osn + ci * osc + (int64_t)p * osp + 4 * j;
  alignas(8) T o0[4], o1[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    o0[k] = vmax(vmax(hm[0][k], hm[1][k]), hm[2][k]);
    o1[k] = vmax(vmax(hm[2][k], hm[3][k]), hm[4][k]);
  }
  *reinterpret_cast<uint2 *>(orow) = *reinterpret_cast<uint2 *>(o0);
  if (p + 1 < P) *reinterpret_cast<uint2 *>(orow + osp) = *reinterpret_cast<uint2 *>(o1);
}

template <typename T>
inline void launch_vec(const T *in, T *out, int64_t n, int64_t c, int64_t h, int64_t w, const int64_t *is,
                       int64_t P, int64_t Q, const int64_t *os, cudaStream_t stream) {
  if constexpr (sizeof(T) == 2) {
    const int pairs_per_plane = (int)((P + 1) / 2);
    const int64_t total_pairs = n * c * pairs_per_plane;
    const int64_t blocks = (total_pairs + 31) / 32;
    launch_overlapped(max_pool2d_3x3s2p1_vec_kernel<T>, dim3((unsigned)blocks), dim3(256), 0, stream, in, out, (int)c,
                      (int)h, (int)w, (int)P, (int)Q, is[0], is[1], is[2], os[0], os[1], os[2], pairs_per_plane,
                      total_pairs);  // a failed launch is read by the caller's launch_status()
  }
}

template <typename T, int WH, int WW, int SH, int SW>
inline void launch_pairs(const T *in, T *out, int64_t n, int64_t c, int64_t h, int64_t w, const int64_t *is,
                         int64_t P, int64_t Q, const int64_t *os, int64_t ph, int64_t pw, cudaStream_t stream) {
  const int64_t pair_rows = (P + 1) / 2;
  const dim3 grid((unsigned)(n * c), (unsigned)((pair_rows + 7) / 8));
  max_pool2d_pairs_kernel<T, WH, WW, SH, SW><<<grid, 256, 0, stream>>>(
      in, out, (int)c, (int)h, (int)w, (int)P, (int)Q, is[0], is[1], is[2], os[0], os[1], os[2], (int)ph, (int)pw);
}

// 2x2 window, stride 2, no padding, 16-bit elements, W % 8 == 0: a thread
// takes 8 columns of input rows 2p and 2p + 1 with two 16-byte loads and writes
// the 4 outputs with one 8-byte store (row 2p + 1 past the input, as the last
// output row of an odd height in ceil mode, reads as -inf).
template <typename T>
__global__ void __launch_bounds__(256)
max_pool2d_2x2s2_vec_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int H, int P, int vecs,
                            int64_t isn, int64_t isc, int64_t ish, int64_t osn, int64_t osc, int64_t osp,
                            int64_t total) {
  using V = typename Pair<T>::V;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int v = (int)(i % vecs);
    const int64_t row = i / vecs;
    const int p = (int)(row % P);
    const int64_t nc = row / P;
    const int ci = (int)(nc % C);
    const int64_t ni = nc / C;
    const T *r0 = in + ni * isn + ci * isc + (int64_t)(2 * p) * ish + 8 * v;
    uint4 a = __ldcs(reinterpret_cast<const uint4 *>(r0));
    uint4 b;
    if (2 * p + 1 < H) {
      b = __ldcs(reinterpret_cast<const uint4 *>(r0 + ish));
    } else {
      const T ninf = neg_inf<T>();
      const unsigned short bits = *reinterpret_cast<const unsigned short *>(&ninf);
      const uint32_t w2 = (uint32_t)bits | ((uint32_t)bits << 16);
      b = make_uint4(w2, w2, w2, w2);
    }
    const V *va = reinterpret_cast<const V *>(&a);
    const V *vb = reinterpret_cast<const V *>(&b);
    alignas(8) T o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const V m = __hmax2(va[k], vb[k]);  // vertical max of columns 2k, 2k + 1
      const T *mm = reinterpret_cast<const T *>(&m);
      o[k] = __hmax(mm[0], mm[1]);
    }
    *reinterpret_cast<uint2 *>(out + ni * osn + ci * osc + (int64_t)p * osp + 4 * v) = *reinterpret_cast<const uint2 *>(o);
  }
}

// 3x3 window, stride 3, no padding (the reference test's default: stride =
// window), 16-bit elements: a thread computes 8 outputs of one output row from
// the 24 input columns under them, three 16-byte loads per input row when the
// segment lies inside the row, element loads with -inf past the row's end or
// below the last input row (ceil mode) otherwise; the 8 outputs leave as one
// 16-byte store when they are all in the row and aligned.
template <typename T>
__global__ void __launch_bounds__(256)
max_pool2d_3x3s3_vec_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int H, int W, int P, int Q,
                            int groups, int64_t isn, int64_t isc, int64_t ish, int64_t osn, int64_t osc,
                            int64_t osp, bool out_vec, int64_t total) {
  const T ninf = neg_inf<T>();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(i % groups);
    const int64_t row = i / groups;
    const int p = (int)(row % P);
    const int64_t nc = row / P;
    const int ci = (int)(nc % C);
    const int64_t ni = nc / C;
    const T *plane = in + ni * isn + ci * isc;
    const int x0 = 24 * g;
    alignas(16) T o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = ninf;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const int y = 3 * p + r;
      if (y >= H) break;
      const T *irow = plane + (int64_t)y * ish + x0;
      alignas(16) T seg[24];
      if (x0 + 24 <= W) {
#pragma unroll
        for (int u = 0; u < 3; ++u) reinterpret_cast<uint4 *>(seg)[u] = __ldcs(reinterpret_cast<const uint4 *>(irow) + u);
      } else {
#pragma unroll
        for (int e = 0; e < 24; ++e) seg[e] = x0 + e < W ? irow[e] : ninf;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = __hmax(o[k], __hmax(__hmax(seg[3 * k], seg[3 * k + 1]), seg[3 * k + 2]));
    }
    T *orow = out + ni * osn + ci * osc + (int64_t)p * osp + 8 * g;
    if (out_vec && 8 * g + 8 <= Q) {
      *reinterpret_cast<uint4 *>(orow) = *reinterpret_cast<const uint4 *>(o);
    } else {
      for (int k = 0; k < 8 && 8 * g + k < Q; ++k) orow[k] = o[k];
    }
  }
}

template <typename T>
inline void launch_3x3s3_vec(const T *in, T *out, int64_t n, int64_t c, int64_t h, int64_t w, const int64_t *is,
                             int64_t P, int64_t Q, const int64_t *os, bool out_vec, cudaStream_t stream) {
  if constexpr (sizeof(T) == 2) {
    const int64_t groups = (Q + 7) / 8;
    const int64_t total = n * c * P * groups;
    int64_t grid = (total + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (grid > cap) grid = cap;
    max_pool2d_3x3s3_vec_kernel<T><<<(unsigned)grid, 256, 0, stream>>>(in, out, (int)c, (int)h, (int)w, (int)P, (int)Q,
                                                                       (int)groups, is[0], is[1], is[2], os[0], os[1],
                                                                       os[2], out_vec, total);
  }
}

template <typename T>
inline void launch_2x2s2_vec(const T *in, T *out, int64_t n, int64_t c, int64_t h, int64_t w, const int64_t *is,
                             int64_t P, const int64_t *os, cudaStream_t stream) {
  if constexpr (sizeof(T) == 2) {
    const int64_t total = n * c * P * (w / 8);
    int64_t grid = (total + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (grid > cap) grid = cap;
    max_pool2d_2x2s2_vec_kernel<T><<<(unsigned)grid, 256, 0, stream>>>(in, out, (int)c, (int)h, (int)P, (int)(w / 8),
                                                                       is[0], is[1], is[2], os[0], os[1], os[2],
                                                                       total);
  }
}

template <typename T, int WH, int WW, int SH, int SW>
inline void launch_rows(const T *in, T *out, int64_t n, int64_t c, int64_t h, int64_t w, const int64_t *is,
                        int64_t P, int64_t Q, const int64_t *os, int64_t wh, int64_t ww, int64_t sh, int64_t sw,
                        int64_t ph, int64_t pw, cudaStream_t stream) {
  const int64_t rows = n * c * P;
  int64_t grid = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 32;
  if (grid > cap) grid = cap;
  max_pool2d_rows_kernel<T, WH, WW, SH, SW><<<(unsigned)grid, 256, 0, stream>>>(
      in, out, (int)c, (int)h, (int)w, (int)P, (int)Q, is[0], is[1], is[2], os[0], os[1], os[2], rows, (int)wh,
      (int)ww, (int)sh, (int)sw, (int)ph, (int)pw);
}

}  // namespace pool
}  // namespace nt

extern "C" int nt_b200_max_pool2d(const void *input, void *output, int64_t n, int64_t c, int64_t h, int64_t w,
                                  const int64_t *input_strides, int64_t out_h, int64_t out_w,
                                  const int64_t *output_strides, int64_t window_h, int64_t window_w,
                                  int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w, int dtype,
                                  void *stream) {
  if (n < 0 || c < 0 || h < 0 || w < 0 || out_h < 0 || out_w < 0) return NT_B200_ERR_INVALID_ARGUMENT;
  if (window_h <= 0 || window_w <= 0 || stride_h <= 0 || stride_w <= 0 || pad_h < 0 || pad_w < 0 ||
      window_h > 4096 || window_w > 4096 || stride_h > (1 << 30) || stride_w > (1 << 30) || pad_h > (1 << 30) ||
      pad_w > (1 << 30))
    return NT_B200_ERR_INVALID_ARGUMENT;
  if (!nt::is_float_dtype(dtype)) return NT_B200_ERR_UNSUPPORTED_DTYPE;
  if (n * c * out_h * out_w == 0) return 0;
  if (!input || !output || !input_strides || !output_strides) return NT_B200_ERR_INVALID_ARGUMENT;
  // Every output window must start inside the padded input.
  if ((out_h - 1) * stride_h - pad_h >= h || (out_w - 1) * stride_w - pad_w >= w) return NT_B200_ERR_SHAPE_MISMATCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t *is = input_strides, *os = output_strides;
  return NT_DISPATCH_FLOAT(dtype, [&] {
    // The row path keeps the in-plane offsets (y * row stride + x) in 32 bits.
    const bool int32_ok = h < (1 << 30) && w < (1 << 30) && out_h < (1 << 30) && out_w < (1 << 30) &&
                          c < (1 << 30) && (h + 1) * (is[2] < 0 ? -is[2] : is[2]) < (1LL << 31);
    const bool grid_ok = n * c < (1LL << 31) && (out_h + 15) / 16 < 65535;
    if (is[3] == 1 && os[3] == 1 && int32_ok && h > 0 && w > 0 && grid_ok) {
      using T = scalar_t;
      const T *in = static_cast<const T *>(input);
      T *out = static_cast<T *>(output);
      const bool pair_aligned = w % 2 == 0 && is[2] % 2 == 0 && is[1] % 2 == 0 && is[0] % 2 == 0 &&
                                (reinterpret_cast<uintptr_t>(input) % (2 * sizeof(T))) == 0;
      const bool vec_ok = sizeof(T) == 2 && w <= 64 && w % 8 == 0 && out_w % 4 == 0 && out_w * 2 <= w + 1 &&
                          is[2] % 8 == 0 && is[1] % 8 == 0 && is[0] % 8 == 0 && os[2] % 4 == 0 && os[1] % 4 == 0 &&
                          os[0] % 4 == 0 && (reinterpret_cast<uintptr_t>(input) & 15u) == 0 &&
                          (reinterpret_cast<uintptr_t>(output) & 7u) == 0;
      if (window_h == 3 && window_w == 3 && stride_h == 2 && stride_w == 2 && pad_h == 1 && pad_w == 1 && vec_ok) {
        nt::pool::launch_vec<T>(in, out, n, c, h, w, is, out_h, out_w, os, s);
      } else if (window_h == 3 && window_w == 3 && stride_h == 2 && stride_w == 2 && pad_h == 1 && pad_w == 1 &&
                 pair_aligned) {
        const dim3 grid((unsigned)(n * c), (unsigned)(((out_h + 1) / 2 + 15) / 16));
        nt::pool::max_pool2d_3x3s2p1_kernel<T><<<grid, 256, 0, s>>>(in, out, (int)c, (int)h, (int)w, (int)out_h,
                                                                    (int)out_w, is[0], is[1], is[2], os[0], os[1],
                                                                    os[2]);
      } else if (window_h == 3 && window_w == 3 && stride_h == 2 && stride_w == 2)
        nt::pool::launch_pairs<T, 3, 3, 2, 2>(in, out, n, c, h, w, is, out_h, out_w, os, pad_h, pad_w, s);
      else if (sizeof(T) == 2 && window_h == 2 && window_w == 2 && stride_h == 2 && stride_w == 2 && pad_h == 0 &&
               pad_w == 0 && w % 8 == 0 && out_w * 2 == w && is[2] % 8 == 0 && is[1] % 8 == 0 && is[0] % 8 == 0 &&
               os[2] % 4 == 0 && os[1] % 4 == 0 && os[0] % 4 == 0 &&
               (reinterpret_cast<uintptr_t>(input) & 15u) == 0 && (reinterpret_cast<uintptr_t>(output) & 7u) == 0) {
        nt::pool::launch_2x2s2_vec<T>(in, out, n, c, h, w, is, out_h, os, s);
      }
      else if (sizeof(T) == 2 && window_h == 3 && window_w == 3 && stride_h == 3 && stride_w == 3 && pad_h == 0 &&
               pad_w == 0 && is[2] % 8 == 0 && is[1] % 8 == 0 && is[0] % 8 == 0 &&
               (reinterpret_cast<uintptr_t>(input) & 15u) == 0)
        nt::pool::launch_3x3s3_vec<T>(in, out, n, c, h, w, is, out_h, out_w, os,
                                      os[2] % 8 == 0 && os[1] % 8 == 0 && os[0] % 8 == 0 &&
                                          (reinterpret_cast<uintptr_t>(output) & 15u) == 0,
                                      s);
      else if (window_h == 3 && window_w == 3 && stride_h == 3 && stride_w == 3)
        nt::pool::launch_pairs<T, 3, 3, 3, 3>(in, out, n, c, h, w, is, out_h, out_w, os, pad_h, pad_w, s);
      else if (window_h == 2 && window_w == 2 && stride_h == 2 && stride_w == 2)
        nt::pool::launch_pairs<T, 2, 2, 2, 2>(in, out, n, c, h, w, is, out_h, out_w, os, pad_h, pad_w, s);
      else
        nt::pool::launch_rows<T, 0, 0, 0, 0>(in, out, n, c, h, w, is, out_h, out_w, os, window_h, window_w,
                                              stride_h, stride_w, pad_h, pad_w, s);
      return nt::launch_status();
    }
    const int64_t total = n * c * out_h * out_w;
    const int threads = 256;
    int64_t grid = (total + threads - 1) / threads;
    const int64_t cap = (int64_t)nt::sm_count() * 16;
    if (grid > cap) grid = cap;
    nt::pool::max_pool2d_kernel<scalar_t><<<(unsigned)grid, threads, 0, s>>>(
        static_cast<const scalar_t *>(input), static_cast<scalar_t *>(output), n, c, h, w, is[0], is[1], is[2],
        is[3], out_h, out_w, os[0], os[1], os[2], os[3], (int)window_h, (int)window_w, (int)stride_h,
        (int)stride_w, (int)pad_h, (int)pad_w);
    return nt::launch_status();
  });
}
