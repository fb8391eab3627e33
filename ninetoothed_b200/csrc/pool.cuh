// 2-D max pooling (the reference's `max_pool2d` arrangement/application,
// tests/test_max_pool2d.py:13-36, and its padded stride-2 variant).
//
// Window positions outside the input are skipped, which is the same as the
// reference's `other=-inf` fill for a max.  The result is an element of the
// input, so it is bit-exact.  One thread per output element, with consecutive
// threads on consecutive output columns: the window rows a warp reads are
// contiguous runs of the input row, and the overlap between neighbouring
// windows is served from L1.
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

// Plane-tiled path for planes with unit column stride: a CTA stages the input
// rows that a band of output rows needs in shared memory (16-byte vector loads
// when the band is aligned, so every input byte is read from HBM once) and
// computes the band's outputs from there with 32-bit index math.
constexpr int kPlaneThreads = 256;
constexpr int kPlaneSmemBytes = 32 * 1024;

template <typename T>
__global__ void __launch_bounds__(kPlaneThreads)
max_pool2d_plane_kernel(const T *__restrict__ in, T *__restrict__ out, int c, int h, int w, int64_t isn,
                        int64_t isc, int64_t ish, int out_h, int out_w, int64_t osn, int64_t osc, int64_t osh,
                        int64_t osw, int wh, int ww, int sh, int sw, int ph, int pw, int band, int bands) {
  __shared__ __align__(16) unsigned char smem_raw[kPlaneSmemBytes];
  T *tile = reinterpret_cast<T *>(smem_raw);
  const int64_t plane = blockIdx.x / bands;
  const int band_idx = blockIdx.x % bands;
  const int ni = (int)(plane / c), ci = (int)(plane % c);
  const int p0 = band_idx * band;
  const int p1 = min(p0 + band, out_h);
  const int y0 = max(p0 * sh - ph, 0);
  const int y1 = min((p1 - 1) * sh - ph + wh, h);  // exclusive
  const int rows = y1 - y0;
  const T *src = in + ni * isn + ci * isc + (int64_t)y0 * ish;
  const int count = rows * w;
  constexpr int E = 16 / sizeof(T);
  const bool packed = ish == w && (reinterpret_cast<uintptr_t>(src) % 16) == 0 && (count % E) == 0;
  if (packed) {
    const int4 *v = reinterpret_cast<const int4 *>(src);
    int4 *t = reinterpret_cast<int4 *>(tile);
    for (int i = threadIdx.x; i < count / E; i += kPlaneThreads) t[i] = __ldcs(v + i);
  } else {
    for (int i = threadIdx.x; i < count; i += kPlaneThreads) {
      const int r = i / w, x = i - r * w;
      tile[i] = src[(int64_t)r * ish + x];
    }
  }
  __syncthreads();
  T *dst = out + ni * osn + ci * osc;
  const int outputs = (p1 - p0) * out_w;
  for (int i = threadIdx.x; i < outputs; i += kPlaneThreads) {
    const int pp = p0 + i / out_w, q = i % out_w;
    const int ys = pp * sh - ph, xs = q * sw - pw;
    float m = -INFINITY;
    for (int r = 0; r < wh; ++r) {
      const int y = ys + r;
      if (y < 0 || y >= h) continue;
      const T *row = tile + (y - y0) * w;
      for (int s2 = 0; s2 < ww; ++s2) {
        const int x = xs + s2;
        if (x < 0 || x >= w) continue;
        const float v = to_f(row[x]);
        m = v > m ? v : m;
      }
    }
    dst[pp * osh + q * osw] = from_f<T>(m);
  }
}

// Output rows per CTA so that the staged input band fits kPlaneSmemBytes;
// 0 when even one output row does not fit.
inline int plane_band(int64_t out_h, int64_t w, int64_t wh, int64_t sh, int elem) {
  const int64_t row_bytes = w * elem;
  if (row_bytes <= 0) return 0;
  const int64_t max_rows = kPlaneSmemBytes / row_bytes;
  if (max_rows < wh) return 0;
  int64_t band = (max_rows - wh) / sh + 1;
  if (band > out_h) band = out_h;
  return (int)band;
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
    const int band = nt::pool::plane_band(out_h, w, window_h, stride_h, (int)sizeof(scalar_t));
    const bool int32_ok = h < (1 << 30) && w < (1 << 30) && out_h < (1 << 30) && out_w < (1 << 30) &&
                          h * w < (1LL << 31) && out_h * out_w < (1LL << 31);
    if (is[3] == 1 && band > 0 && int32_ok) {
      const int64_t bands = (out_h + band - 1) / band;
      const int64_t grid = n * c * bands;
      if (grid < (1LL << 31)) {
        nt::pool::max_pool2d_plane_kernel<scalar_t><<<(unsigned)grid, nt::pool::kPlaneThreads, 0, s>>>(
            static_cast<const scalar_t *>(input), static_cast<scalar_t *>(output), (int)c, (int)h, (int)w, is[0],
            is[1], is[2], (int)out_h, (int)out_w, os[0], os[1], os[2], os[3], (int)window_h, (int)window_w,
            (int)stride_h, (int)stride_w, (int)pad_h, (int)pad_w, band, (int)bands);
        return nt::launch_status();
      }
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
