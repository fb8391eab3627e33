// tcgen05 tensor-core GEMM for the reference's blocked-linalg programs:
// matmul (tests/test_matmul.py:14-47) and addmm (tests/test_addmm.py:13-38).
//
// Design (one CTA per SM, persistent):
//   warp 0      TMA producer: A tile 128x64 and B tile 64x256 per k-block into a
//               4-stage shared-memory ring (128-byte swizzle), one mbarrier pair
//               (full/empty) per stage;
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and
//               issues tcgen05.mma (M=128, N=256, K=16) from one thread;
//               tcgen05.commit releases smem stages and publishes finished
//               accumulators;
//   warps 2-5   epilogue: tcgen05.ld of one accumulator row per thread, the
//               application's cast chain, 16-byte global stores; it drains one
//               accumulator while the MMA warp fills the other.
// Output tiles are walked in groups of 16 row-tiles so that the A and B panels
// of a wave of 148 CTAs stay in L2.  Every mbarrier wait is bounded in time.
#pragma once

#include <cuda.h>
#include <cuda_fp8.h>
#include "common.cuh"
#include "ptx.cuh"

namespace nt {
namespace tc {

constexpr int kNotEligible = -1;

// kConvPool: conv2d whose output also feeds a fused 3x3 / stride 2 / padding 1
// max pool (CTA-pair kernel only).
enum class Epilogue { kMatmul, kAddmm, kConv, kConvPool };
__host__ __device__ constexpr bool is_conv(Epilogue e) { return e == Epilogue::kConv || e == Epilogue::kConvPool; }

struct GemmProblem {
  const void *a, *b, *bias;
  void *out;
  int64_t M, N, K;
  int64_t sam, sak, sbk, sbn, sim, sin, som, son;
  float beta, alpha;
};

// Output side of conv2d + max_pool2d (3x3, stride 2, padding 1) fused in the
// CTA-pair conv epilogue: pooled output, its strides, extents and the
// per-(image, channel tile, pool row) counters (workspace, zeroed per call).
struct PoolFusion {
  void *out;
  int64_t os[4];
  int P2, Q2;
  int *counters;
};

struct ConvProblem {
  const void *input, *filter;
  void *output;
  int64_t n, c, h, w, k, r, s, pad_h, pad_w, P, Q;
  int64_t is[4], fs[4], os[4];
};

// ------------------------------------------------------------------ host: tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn();

using EncodeIm2colFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const int *, const int *, cuuint32_t, cuuint32_t,
                                    const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeIm2colFn encode_im2col_fn();

// 2-D tensor map over a matrix with a contiguous inner dimension.
inline bool make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                         uint64_t outer, uint64_t outer_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {outer_stride_elems * (uint64_t)elem_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T> constexpr CUtensorMapDataType tmap_dtype();
template <> constexpr CUtensorMapDataType tmap_dtype<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }
template <> constexpr CUtensorMapDataType tmap_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <> constexpr CUtensorMapDataType tmap_dtype<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <> constexpr CUtensorMapDataType tmap_dtype<__nv_fp8_e4m3>() { return CU_TENSOR_MAP_DATA_TYPE_UINT8; }
template <> constexpr CUtensorMapDataType tmap_dtype<__nv_fp8_e5m2>() { return CU_TENSOR_MAP_DATA_TYPE_UINT8; }

template <typename T> __host__ __device__ constexpr uint32_t umma_format();
template <> __host__ __device__ constexpr uint32_t umma_format<__half>() { return 0; }
template <> __host__ __device__ constexpr uint32_t umma_format<__nv_bfloat16>() { return 1; }
template <> __host__ __device__ constexpr uint32_t umma_format<float>() { return 0; }
template <> __host__ __device__ constexpr uint32_t umma_format<__nv_fp8_e4m3>() { return 0; }
template <> __host__ __device__ constexpr uint32_t umma_format<__nv_fp8_e5m2>() { return 1; }

// ------------------------------------------------------------------ kernel
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, GROUP_M = 16;
constexpr int A_STAGE_BYTES = BM * 128;  // 16 KB: 128 rows of one 128-byte swizzle row
constexpr int B_STAGE_BYTES = BN * 128;  // 32 KB
// A k-block is one 128-byte row of K elements: 64 for 16-bit, 128 for 8-bit
// types; one MMA instruction consumes 32 bytes of K (16 or 32 elements).
template <typename T> __host__ __device__ constexpr int kblock() { return 128 / (int)sizeof(T); }
template <typename T> __host__ __device__ constexpr int mma_k() { return 32 / (int)sizeof(T); }
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + 1024 /*align*/ + 256 /*barriers*/;

struct Params {
  int64_t M, N, K;
  void *out;
  int64_t som, son;
  const void *bias;
  int64_t sim, sin;
  float beta, alpha;  // rounded to TI and float16 (addmm_value)
  int tiles_m, tiles_n, num_kb;
  // conv2d implicit GEMM (EPI == kConv): an m-block is 128 consecutive
  // positions pos = p * Wp + q of one image on the W-padded grid (Wp = W +
  // 2 pad_w columns; positions with q >= Q are computed and dropped); k-block
  // kb = (r, s, channel block cb).
  int conv_c_blocks, conv_s, conv_pad_h, conv_wp, conv_tiles_img, conv_P, conv_Q;
  int64_t conv_osn, conv_osk, conv_osp, conv_osq;
  // conv_flat (CTA-pair kConv only): m-blocks tile the batch's output pixels
  // as one range f = image * conv_pwp + p * Q + q (conv_pwp = P * Q, conv_wp
  // = Q: no padding columns), and A is loaded by im2col-mode TMA from the
  // unpadded NHWC input; conv_n images
  int conv_flat, conv_pwp, conv_n, conv_pad_w;
  // fused max pool (EPI == kConvPool): the conv output above is the pool's
  // input (a dense NCHW workspace); pool rows of P2 x Q2, and one counter per
  // (image, output-channel tile, pool row)
  void *pool_out;
  int64_t pool_osn, pool_osk, pool_osi, pool_osj;
  int pool_P, pool_Q;
  int *pool_counters;
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int &mb, int &nb,
                                            int group_m = GROUP_M) {
  const int per_group = group_m * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * group_m;
  const int gsize = min(tiles_m - first_m, group_m);
  const int in_group = tile % per_group;
  mb = first_m + in_group % gsize;
  nb = in_group / gsize;
}

template <typename TO>
__device__ __forceinline__ void store_row_chunk(TO *dst, const float (&v)[32], bool full, int valid) {
  if (full) {
    if constexpr (sizeof(TO) == 2) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        alignas(16) TO tmp[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) tmp[e] = from_f<TO>(v[i * 8 + e]);
        *reinterpret_cast<int4 *>(dst + i * 8) = *reinterpret_cast<int4 *>(tmp);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float4 *>(dst + i * 4) = make_float4(v[i * 4], v[i * 4 + 1], v[i * 4 + 2], v[i * 4 + 3]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e)
      if (e < valid) dst[e] = from_f<TO>(v[e]);
  }
}

// Epilogue of one accumulator: this warp's 32 TMEM lanes (tile rows
// quarter * 32 + lane) x 256 columns starting at TMEM column `col0`.  Row r of
// the tile is output row row0 + r (matmul, addmm), or position row0 + r
// (= p * Wp + q) of image `img` (conv2d); columns are outputs n0, n0 + 1, ...
template <typename TI, typename TO, Epilogue EPI>
__device__ __forceinline__ void store_accumulator(const Params &prm, uint32_t tmem_base, uint32_t col0, int quarter,
                                                  int lane, int64_t row0, int64_t n0, int img) {
  const int row_in_tile = quarter * 32 + lane;
  const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16) + col0;
  TO *out = static_cast<TO *>(prm.out);
  if constexpr (is_conv(EPI)) {
    // TMEM lane = position p * Wp + q; columns = output channels.
    int pos = (int)row0 + row_in_tile;
    if (prm.conv_flat) {  // row0 is a flat position (< 2^31): split it into image and position
      const int f = (int)row0 + row_in_tile;
      img = f / prm.conv_pwp;
      pos = f - img * prm.conv_pwp;
    }
    const int p = pos / prm.conv_wp, q = pos % prm.conv_wp;
    const bool pix_ok = img < prm.conv_n && p < prm.conv_P && q < prm.conv_Q;
    TO *pix = out + (int64_t)img * prm.conv_osn + (int64_t)p * prm.conv_osp + (int64_t)q * prm.conv_osq;
#pragma unroll 1
    for (int c = 0; c < 256 / 32; ++c) {
      uint32_t raw[32];
      ptx::tmem_ld_32x32b_x32(lane_base + (uint32_t)(c * 32), raw);
      ptx::tmem_ld_wait();
      const int64_t nc = n0 + c * 32;
      if (!pix_ok || nc >= prm.N) continue;
      const int valid = (int)(prm.N - nc < 32 ? prm.N - nc : 32);
      TO *dst = pix + nc * prm.conv_osk;
      if (prm.conv_osk == 1) {  // channels-last output: the pixel's 32 channels are one run
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = round_f16(__uint_as_float(raw[e]));
        store_row_chunk<TO>(dst, v, valid == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0, valid);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (e < valid) dst[e * prm.conv_osk] = from_f<TO>(round_f16(__uint_as_float(raw[e])));
      }
    }
  } else {
    const int64_t m = row0 + row_in_tile;
    const bool row_ok = m < prm.M;
#pragma unroll 1
    for (int c = 0; c < 256 / 32; ++c) {
      uint32_t raw[32];
      ptx::tmem_ld_32x32b_x32(lane_base + (uint32_t)(c * 32), raw);
      ptx::tmem_ld_wait();
      const int64_t nc = n0 + c * 32;
      if (!row_ok || nc >= prm.N) continue;
      const int valid = (int)(prm.N - nc < 32 ? prm.N - nc : 32);
      float v[32];
      if constexpr (EPI == Epilogue::kMatmul) {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = round_f16(__uint_as_float(raw[e]));
      } else if constexpr (EPI == Epilogue::kAddmm) {
        const TI *bias = static_cast<const TI *>(prm.bias) + m * prm.sim + nc * prm.sin;
        alignas(16) TI in_v[32];
        if (valid == 32 && prm.sin == 1 && (reinterpret_cast<uintptr_t>(bias) & 15u) == 0) {
          // the row's 32 inputs are one contiguous run: 16-byte loads
#pragma unroll
          for (int i = 0; i < 32 * (int)sizeof(TI) / 16; ++i)
            reinterpret_cast<int4 *>(in_v)[i] = __ldcs(reinterpret_cast<const int4 *>(bias) + i);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) in_v[e] = e < valid ? bias[e * prm.sin] : from_f<TI>(0.f);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = addmm_value<TI>(prm.beta, prm.alpha, to_f(in_v[e]), __uint_as_float(raw[e]));
      }
      TO *dst = out + m * prm.som + nc * prm.son;
      const bool vec = valid == 32 && prm.son == 1 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
      if (vec || prm.son == 1) {
        store_row_chunk<TO>(dst, v, vec, valid);
      } else {
        for (int e = 0; e < valid; ++e) dst[e * prm.son] = from_f<TO>(v[e]);
      }
    }
  }
}

// Two 16-bit values as one 32-bit word (first in the low half), and back.
template <typename T>
__device__ __forceinline__ uint32_t pack2_16(float a, float b) {
  const T x = from_f<T>(a), y = from_f<T>(b);
  uint16_t ux, uy;
  memcpy(&ux, &x, 2);
  memcpy(&uy, &y, 2);
  return (uint32_t)ux | ((uint32_t)uy << 16);
}
template <typename T>
__device__ __forceinline__ float unpack_16(uint32_t w, int hi) {
  const uint16_t u = (uint16_t)(hi ? (w >> 16) : (w & 0xffffu));
  T x;
  memcpy(&x, &u, 2);
  return to_f(x);
}

// store_accumulator for matmul / addmm with a 16-bit, row-contiguous output
// (and, for addmm, a row-contiguous input) whose rows start on 16-byte
// boundaries, through a 2 KB shared-memory block per warp: each 32 x 32 chunk
// is written by rows (a thread holds one row after tcgen05.ld) and read back
// by row segments, so a warp's global store covers eight rows x 64 contiguous
// bytes instead of 32 rows x 16 bytes (four times fewer store transactions);
// addmm's input chunk comes in the same way, transposed.  Slot c of row r
// sits at 16-byte unit 4 r + ((c + r / 2) mod 4), which keeps both the row
// and the segment passes free of bank conflicts.  Results are those of
// store_accumulator.
template <typename TI, typename TO, Epilogue EPI>
__device__ __forceinline__ void store_accumulator_staged(const Params &prm, uint32_t tmem_base, uint32_t col0,
                                                         int quarter, int lane, int64_t row0, int64_t n0,
                                                         int4 *stage) {
  static_assert(sizeof(TO) == 2 && (EPI == Epilogue::kMatmul || EPI == Epilogue::kAddmm), "16-bit matmul/addmm");
  const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16) + col0;
  const int64_t wrow0 = row0 + quarter * 32;  // this warp's first output row
  TO *out = static_cast<TO *>(prm.out);
  const auto unit = [](int r, int c) { return 4 * r + ((c + (r >> 1)) & 3); };
#pragma unroll 1
  for (int c = 0; c < 256 / 32; ++c) {
    uint32_t raw[32];
    ptx::tmem_ld_32x32b_x32(lane_base + (uint32_t)(c * 32), raw);
    ptx::tmem_ld_wait();
    const int64_t nc = n0 + c * 32;
    if (nc >= prm.N) continue;  // the same in every lane
    const bool full = prm.N - nc >= 32;
    const int64_t m = wrow0 + lane;
    float v[32];
    if constexpr (EPI == Epilogue::kMatmul) {
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = round_f16(__uint_as_float(raw[e]));
    } else {
      float in_v[32];
      if (full) {
        const TI *bias = static_cast<const TI *>(prm.bias) + nc;
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // segments: rows 8i .. 8i + 7, four 16-byte slots each
          const int r = 8 * i + (lane >> 2), slot = lane & 3;
          const int64_t mr = wrow0 + r;
          stage[unit(r, slot)] =
              mr < prm.M ? __ldcs(reinterpret_cast<const int4 *>(bias + mr * prm.sim) + slot) : make_int4(0, 0, 0, 0);
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int4 q = stage[unit(lane, j)];
          const uint32_t w[4] = {(uint32_t)q.x, (uint32_t)q.y, (uint32_t)q.z, (uint32_t)q.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) in_v[j * 8 + e] = unpack_16<TI>(w[e >> 1], e & 1);
        }
        __syncwarp();
      } else {
        const int valid = (int)(prm.N - nc);
        const TI *bias = static_cast<const TI *>(prm.bias) + m * prm.sim + nc * prm.sin;
#pragma unroll
        for (int e = 0; e < 32; ++e) in_v[e] = (e < valid && m < prm.M) ? to_f(bias[e * prm.sin]) : 0.f;
      }
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] = addmm_value<TI>(prm.beta, prm.alpha, in_v[e], __uint_as_float(raw[e]));
    }
    if (full) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        stage[unit(lane, j)] =
            make_int4((int)pack2_16<TO>(v[j * 8 + 0], v[j * 8 + 1]), (int)pack2_16<TO>(v[j * 8 + 2], v[j * 8 + 3]),
                      (int)pack2_16<TO>(v[j * 8 + 4], v[j * 8 + 5]), (int)pack2_16<TO>(v[j * 8 + 6], v[j * 8 + 7]));
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 8 * i + (lane >> 2), slot = lane & 3;
        const int64_t mr = wrow0 + r;
        if (mr < prm.M) *(reinterpret_cast<int4 *>(out + mr * prm.som + nc) + slot) = stage[unit(r, slot)];
      }
      __syncwarp();
    } else if (m < prm.M) {
      const int valid = (int)(prm.N - nc);
      for (int e = 0; e < valid; ++e) out[m * prm.som + (nc + e) * prm.son] = from_f<TO>(v[e]);
    }
  }
}

template <typename TI, typename TO, Epilogue EPI, bool B_MN_MAJOR>
__global__ void __launch_bounds__(THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, Params prm) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  const uint32_t a_base = base;
  const uint32_t b_base = base + STAGES * A_STAGE_BYTES;
  uint8_t *ctrl = smem + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES);
  const uint32_t ctrl_addr = ptx::smem_u32(ctrl);
  // barriers: full[S], empty[S], tfull[2], tempty[2]; then tmem base and abort flag
  auto full_bar = [&](int s) { return ctrl_addr + 8u * s; };
  auto empty_bar = [&](int s) { return ctrl_addr + 8u * (STAGES + s); };
  auto tfull_bar = [&](int b) { return ctrl_addr + 8u * (2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return ctrl_addr + 8u * (2 * STAGES + 2 + b); };
  volatile uint32_t *tmem_base_ptr = reinterpret_cast<volatile uint32_t *>(ctrl + 8 * (2 * STAGES + 4));
  volatile int *abort_flag = reinterpret_cast<volatile int *>(ctrl + 8 * (2 * STAGES + 4) + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(tfull_bar(b), 1);
      ptx::mbar_init(tempty_bar(b), 128);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(const_cast<uint32_t *>(tmem_base_ptr)), TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_base_ptr;

  const int num_tiles = prm.tiles_m * prm.tiles_n;
  const int num_kb = prm.num_kb;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, prm.tiles_m, prm.tiles_n, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t fb = full_bar(stage);
          ptx::mbar_arrive_expect_tx(fb, A_STAGE_BYTES + B_STAGE_BYTES);
          const int k0 = kb * kblock<TI>();
          if constexpr (is_conv(EPI)) {
            // A: 128 consecutive rows x 64 channels of the W-padded NHWC input
            // of one image, shifted by filter tap (r, s): position pos reads
            // row pos + (r - pad_h) * Wp + s.  Rows above or below the image
            // (negative or >= H * Wp) read as zero, which is the H padding;
            // the W padding is stored as zero columns.
            // B: 256 output channels x 64 input channels of the KRSC filter.
            const int cb = kb % prm.conv_c_blocks, rs = kb / prm.conv_c_blocks;
            const int r = rs / prm.conv_s, sx = rs % prm.conv_s;
            const int img = mb / prm.conv_tiles_img, pos0 = (mb % prm.conv_tiles_img) * BM;
            ptx::tma_load_3d(a_base + stage * A_STAGE_BYTES, &tmap_a, fb, cb * BK,
                             pos0 + (r - prm.conv_pad_h) * prm.conv_wp + sx, img);
            ptx::tma_load_3d(b_base + stage * B_STAGE_BYTES, &tmap_b, fb, cb * BK, rs, n0);
          } else {
          ptx::tma_load_2d(a_base + stage * A_STAGE_BYTES, &tmap_a, fb, k0, m0);
          if constexpr (B_MN_MAJOR) {
#pragma unroll
            for (int j = 0; j < BN / kblock<TI>(); ++j)
              ptx::tma_load_2d(b_base + stage * B_STAGE_BYTES + j * (kblock<TI>() * 128), &tmap_b, fb,
                               n0 + kblock<TI>() * j, k0);
          } else {
            ptx::tma_load_2d(b_base + stage * B_STAGE_BYTES, &tmap_b, fb, k0, n0);
          }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::f16_idesc(umma_format<TI>(), 0, B_MN_MAJOR ? 1 : 0, BM, BN);  // same
      // bit layout for kind::f8f6f4 (format codes E4M3 = 0, E5M2 = 1)
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1) & 1u;
        if (!ptx::mbar_wait(tempty_bar(buf), use ^ 1u, abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!ptx::mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t a_addr = a_base + stage * A_STAGE_BYTES;
          const uint32_t b_addr = b_base + stage * B_STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 4 x 32 bytes of K
            const uint64_t a_desc = ptx::sw128_desc(a_addr + kk * 32, 16, 1024);
            uint64_t b_desc;
            if constexpr (B_MN_MAJOR)
              b_desc = ptx::sw128_desc(b_addr + kk * mma_k<TI>() * 128, kblock<TI>() * 128, 1024);
            else
              b_desc = ptx::sw128_desc(b_addr + kk * 32, 16, 1024);
            if constexpr (sizeof(TI) == 1)
              ptx::mma_f8_ss(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
            else
              ptx::mma_f16_ss(d_tmem, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          ptx::mma_commit(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) ptx::mma_commit(tfull_bar(buf));
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1) & 1u;
      if (!ptx::mbar_wait_warp(tfull_bar(buf), use, abort_flag)) break;
      ptx::tc_fence_after();
      int mb, nb;
      tile_coords(tile, prm.tiles_m, prm.tiles_n, mb, nb);
      if constexpr (is_conv(EPI))
        store_accumulator<TI, TO, EPI>(prm, tmem_base, (uint32_t)(buf * BN), quarter, lane,
                                       (int64_t)(mb % prm.conv_tiles_img) * BM, (int64_t)nb * BN,
                                       mb / prm.conv_tiles_img);
      else
        store_accumulator<TI, TO, EPI>(prm, tmem_base, (uint32_t)(buf * BN), quarter, lane, (int64_t)mb * BM,
                                       (int64_t)nb * BN, 0);
      ptx::tc_fence_before();
      ptx::mbar_arrive(tempty_bar(buf));
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm

// ------------------------------------------------------------------ CTA-pair kernel
// The same GEMM on CTA pairs (thread-block clusters of 2) with tcgen05
// .cta_group::2: a pair computes a 256 x 256 output tile with M = 256 MMAs
// issued by the even CTA.  Each CTA stages its own 128 rows of A and its half
// (128 columns) of B, so every operand byte crosses from L2 once per pair tile
// instead of B being fetched by two independent 128-row tiles: 32 KB per CTA
// per 64-element k-block instead of 48 KB, which lets six stages fit in
// shared memory.  Both CTAs' loads complete on the even CTA's `full` barrier;
// the MMA commits release the stage (and publish the accumulator) in both
// CTAs; both CTAs' epilogue warps release the accumulator on the even CTA's
// `tempty` barrier.
namespace gemm2 {

constexpr int BM = 128;      // A rows per CTA; the pair tile is 2 * BM = 256 rows
constexpr int BN = 256;      // output columns of a pair tile
constexpr int BN_CTA = 128;  // B rows (output columns) staged per CTA
constexpr int STAGES = 7;
constexpr int A_STAGE_BYTES = BM * 128;      // 16 KB
constexpr int B_STAGE_BYTES = BN_CTA * 128;  // 16 KB
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;
// kConvPool adds POOL_WARPS pool warps (warps 6..) fed by a ring of RING work
// cells in shared memory; the control block holds the barriers, the ring's
// counters (from byte 152) and the cells (from byte 256).
constexpr int POOL_WARPS = 6;
constexpr int RING = 128;
constexpr int CTRL_BYTES = 256 + 8 * RING;
constexpr int SMEM_BYTES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + 1024 /*align*/ + CTRL_BYTES;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
static_assert(8 * (2 * STAGES + 4) + 8 + 12 <= 256, "control block");
// MB = 128-row blocks of A per CTA.  MB = 1: 256 x 256 pair tiles, 7-stage ring,
// two accumulators in TMEM (the epilogue of one tile overlaps the next).
// MB = 2: 512 x 256 pair tiles, each staged B block feeding two MMAs (one per
// A block), 4-stage ring of 48 KB, one accumulator set of 2 x 256 columns
// drained by two epilogue warpgroups side by side: a third less L2 -> SM
// traffic per FLOP.
template <int MB>
struct PairCfg {
  static constexpr int STAGES = MB == 1 ? 7 : 4;
  static constexpr int A_STAGE_BYTES = MB * BM * 128;
  static constexpr int NBUF = MB == 1 ? 2 : 1;  // accumulator sets of MB x BN columns
  static constexpr int GROUP_M = 16 / MB;       // raster groups of 4096 A rows
  // MB = 2: a 2 KB output staging block per epilogue warp after the control
  // block (store_accumulator_staged)
  static constexpr int EPI_STAGE_BYTES = MB == 2 ? 8 * 2048 : 0;
  static constexpr int SMEM_BYTES =
      STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + 1024 /*align*/ + CTRL_BYTES + EPI_STAGE_BYTES;
  static_assert(NBUF * MB * BN <= TMEM_COLS, "TMEM columns");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

// MB = 2 doubles the epilogue: warps 2-5 drain A block 0's accumulator,
// warps 6-9 A block 1's, side by side.
__host__ __device__ constexpr int threads_for(Epilogue e, int mb = 1) {
  return e == Epilogue::kConvPool ? THREADS + 32 * POOL_WARPS : THREADS + (mb - 1) * 128;
}

using gemm::Params;
using gemm::kblock;
using gemm::mma_k;

// Fused 3x3 / stride 2 / padding 1 max pool (EPI == kConvPool).
//
// Pool row i of image `img` and channel tile nb (256 channels) reads conv rows
// 2i - 1 .. 2i + 1; the 32-position blocks that cover them are stored by
// different epilogue warps, CTAs and tiles.  After storing its block, an
// epilogue warp counts it on every pool row it overlaps (one counter per
// image, channel tile and pool row, in global memory); the block whose count
// completes a row hands the row, as one work cell per 32 channels, to the pool
// warps of its own CTA through a ring in shared memory.  No warp waits for
// another CTA, and the epilogue only waits when the ring is full.  The conv
// output is read back with L1-bypassing loads: L1 is not coherent with the
// other SMs' stores.
//
// The ring is a bounded multi-producer multi-consumer queue of RING cells
// (sequence number, work code): the producer of position t waits for cell
// t % RING to carry sequence t, writes the code and publishes t + 1; the
// consumer of t waits for t + 1, reads the code and frees the cell with
// t + RING.  Positions are handed out by atomics on `tail` (producers) and
// `head` (consumers).  A work code is 8 * (pool-row counter index) + part.
struct PoolRing {
  int *tail, *head, *epi_done;
  int *cells;  // RING x {sequence, code}
};

__device__ __forceinline__ int ld_volatile_shared(const int *p) { return *reinterpret_cast<const volatile int *>(p); }

// Epilogue side: count the warp's block [wpos, wpos + 32) of image `img` and
// push the pool rows it completes.  Lane 0 only.
__device__ __forceinline__ void pool_count_and_push(const Params &prm, const PoolRing &ring, int img, int wpos,
                                                    int nb, volatile int *abort_flag) {
  const int Wp = prm.conv_wp, P = prm.conv_P, P2 = prm.pool_P;
  const int lo = wpos, hi = min(wpos + 32, P * Wp);
  if (lo >= hi) return;
  __threadfence();  // the warp's stores of this block are visible device-wide before they are counted
  const int p_lo = lo / Wp, p_hi = (hi - 1) / Wp;
  const int i_first = max(0, p_lo / 2 - 1), i_last = min(P2 - 1, (p_hi + 1) / 2);
  const int64_t row0 = ((int64_t)img * prm.tiles_n + nb) * P2;
  const int64_t left = (prm.N - (int64_t)nb * 256 + 31) / 32;
  const int parts = left < 8 ? (int)left : 8;
  for (int i = i_first; i <= i_last; ++i) {
    const int r_lo = max(0, 2 * i - 1), r_hi = min(P - 1, 2 * i + 1);
    if (r_hi < p_lo || r_lo > p_hi) continue;
    const int b_lo = r_lo * Wp, b_hi = (r_hi + 1) * Wp;    // the pool row's input positions
    const int required = (b_hi - 1) / 32 - b_lo / 32 + 1;  // 32-position blocks covering them
    if (atomicAdd(prm.pool_counters + row0 + i, 1) != required - 1) continue;
    __threadfence();  // the other blocks' stores are visible to this CTA's pool warps from here on
    const int pos0 = atomicAdd(ring.tail, parts);
    for (int j = 0; j < parts; ++j) {
      const int pos = pos0 + j;
      int *cell = ring.cells + 2 * (pos % RING);
      const uint64_t t0 = ptx::global_timer_ns();
      bool ok = true;
      for (uint32_t it = 0; ld_volatile_shared(cell) != pos; ++it) {
        if (*abort_flag) { ok = false; break; }
        if ((it & 15u) == 15u && ptx::global_timer_ns() - t0 > ptx::kWaitLimitNs) {
          *abort_flag = 1;
          record_error(NT_B200_ERR_DEVICE_TIMEOUT);
          ok = false;
          break;
        }
        __nanosleep(64);
      }
      if (!ok) return;
      cell[1] = (int)((row0 + i) * 8 + j);
      __threadfence_block();
      *reinterpret_cast<volatile int *>(cell) = pos + 1;
    }
  }
}

// One work cell: pool row i, channels [256 nb + 32 part, + 32) of image img.
// 8 lanes per channel (lane v holds conv columns [8v, 8v + 8) of the three
// input rows and takes column 8v - 1 from lane v - 1), 4 channels per pass,
// all 8 passes' loads in flight at once; lane v writes pool columns
// [4v, 4v + 4) with one 8-byte store.  The host only fuses when Q % 8 == 0,
// Q <= 64 and the pooled rows take 8-byte stores.
template <typename TO>
__device__ __forceinline__ void pool_part(const Params &prm, int img, int nb, int i, int part, int lane) {
  const int P = prm.conv_P, Q = prm.conv_Q;
  const int v = lane & 7, g = lane >> 3;
  const bool col_ok = v < Q / 8;
  const TO ninf = from_f<TO>(-INFINITY);
  const unsigned short ninf_bits = *reinterpret_cast<const unsigned short *>(&ninf);
  const uint32_t ninf2 = (uint32_t)ninf_bits | ((uint32_t)ninf_bits << 16);
  const TO *ybase = static_cast<const TO *>(prm.out) + (int64_t)img * prm.conv_osn;
  TO *zbase = static_cast<TO *>(prm.pool_out) + (int64_t)img * prm.pool_osn;
  const int64_t k0 = (int64_t)nb * 256 + part * 32;
  int4 raw[8][3];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int64_t k = k0 + 4 * u + g;
#pragma unroll
    for (int rr = 0; rr < 3; ++rr) {
      const int r = 2 * i - 1 + rr;
      raw[u][rr] = make_int4((int)ninf2, (int)ninf2, (int)ninf2, (int)ninf2);
      if (col_ok && k < prm.N && r >= 0 && r < P)
        raw[u][rr] = __ldcg(reinterpret_cast<const int4 *>(ybase + k * prm.conv_osk + (int64_t)r * prm.conv_osp) + v);
    }
  }
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int64_t k = k0 + 4 * u + g;
    TO vm[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const TO *r0 = reinterpret_cast<const TO *>(&raw[u][0]);
      const TO *r1 = reinterpret_cast<const TO *>(&raw[u][1]);
      const TO *r2 = reinterpret_cast<const TO *>(&raw[u][2]);
      vm[e] = __hmax(__hmax(r0[e], r1[e]), r2[e]);
    }
    // conv column 8v - 1 is lane v - 1's last element (padding for v = 0)
    const unsigned short last = *reinterpret_cast<const unsigned short *>(&vm[7]);
    const unsigned short prev = (unsigned short)__shfl_up_sync(0xffffffffu, (unsigned)last, 1, 8);
    TO left;
    *reinterpret_cast<unsigned short *>(&left) = prev;
    if (v == 0) left = ninf;
    alignas(8) TO o[4];
#pragma unroll
    for (int oo = 0; oo < 4; ++oo) o[oo] = __hmax(__hmax(oo == 0 ? left : vm[2 * oo - 1], vm[2 * oo]), vm[2 * oo + 1]);
    if (col_ok && k < prm.N)
      *reinterpret_cast<uint2 *>(zbase + k * prm.pool_osk + (int64_t)i * prm.pool_osi + 4 * v) =
          *reinterpret_cast<const uint2 *>(o);
  }
}

// Pool warp: takes ring positions one at a time until the CTA's 4 epilogue
// warps have finished and every pushed position is taken.  Waits are bounded.
template <typename TO>
__device__ __forceinline__ void pool_worker(const Params &prm, const PoolRing &ring, int lane,
                                            volatile int *abort_flag) {
  for (;;) {
    int code = -1;
    if (lane == 0) {
      const uint64_t t0 = ptx::global_timer_ns();
      const int pos = atomicAdd(ring.head, 1);
      int *cell = ring.cells + 2 * (pos % RING);
      for (uint32_t it = 0;; ++it) {
        if (ld_volatile_shared(cell) == pos + 1) {
          __threadfence_block();
          code = ld_volatile_shared(cell + 1);
          __threadfence_block();
          *reinterpret_cast<volatile int *>(cell) = pos + RING;
          break;
        }
        if (ld_volatile_shared(ring.epi_done) == 4) {
          __threadfence_block();
          if (ld_volatile_shared(ring.tail) <= pos) break;  // nothing more will be pushed here
        }
        if (*abort_flag) break;
        if ((it & 15u) == 15u && ptx::global_timer_ns() - t0 > ptx::kWaitLimitNs) {
          *abort_flag = 1;
          record_error(NT_B200_ERR_DEVICE_TIMEOUT);
          break;
        }
        __nanosleep(128);
      }
      if (code >= 0) __threadfence();  // pairs with the producer's device-wide fence
    }
    code = __shfl_sync(0xffffffffu, code, 0);
    if (code < 0) return;
    const int part = code & 7, row = code >> 3;
    const int i = row % prm.pool_P, t = row / prm.pool_P;
    pool_part<TO>(prm, t / prm.tiles_n, t % prm.tiles_n, i, part, lane);
  }
}

template <typename TI, typename TO, Epilogue EPI, bool B_MN_MAJOR, int MB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_for(EPI, MB), 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 Params prm) {
  static_assert(MB == 1 || !is_conv(EPI), "conv tiles are 256 positions");
  constexpr int STAGES = PairCfg<MB>::STAGES;
  constexpr int A_STAGE_BYTES = PairCfg<MB>::A_STAGE_BYTES;
  constexpr int NBUF = PairCfg<MB>::NBUF;
  constexpr int GROUP = PairCfg<MB>::GROUP_M;
  constexpr int TILE_M = 2 * BM * MB;  // rows of a pair tile
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;  // same offset in both CTAs
  uint8_t *smem = smem_raw + (base - raw_addr);
  const uint32_t a_base = base;
  const uint32_t b_base = base + STAGES * A_STAGE_BYTES;
  uint8_t *ctrl = smem + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES);
  const uint32_t ctrl_addr = ptx::smem_u32(ctrl);
  // barriers: full[S] (used on the even CTA), empty[S], tfull[2], tempty[2]
  // (used on the even CTA); then the TMEM base and the abort flag
  auto full_bar = [&](int s) { return ctrl_addr + 8u * s; };
  auto empty_bar = [&](int s) { return ctrl_addr + 8u * (STAGES + s); };
  auto tfull_bar = [&](int b) { return ctrl_addr + 8u * (2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return ctrl_addr + 8u * (2 * STAGES + 2 + b); };
  volatile uint32_t *tmem_base_ptr = reinterpret_cast<volatile uint32_t *>(ctrl + 8 * (2 * STAGES + 4));
  volatile int *abort_flag = reinterpret_cast<volatile int *>(ctrl + 8 * (2 * STAGES + 4) + 4);
  int *ring_words = reinterpret_cast<int *>(ctrl + 8 * (2 * STAGES + 4) + 8);
  const PoolRing ring{ring_words, ring_words + 1, ring_words + 2, reinterpret_cast<int *>(ctrl + 256)};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);   // the even CTA's producer arrives (with both CTAs' bytes)
      ptx::mbar_init(empty_bar(s), 1);  // one MMA commit per use
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(tfull_bar(b), 1);
      ptx::mbar_init(tempty_bar(b), 8 * MB);  // one arrival per epilogue warp of both CTAs
    }
    *abort_flag = 0;
    if constexpr (EPI == Epilogue::kConvPool) {
      *ring.tail = *ring.head = *ring.epi_done = 0;
      for (int c = 0; c < RING; ++c) ring.cells[2 * c] = c;
    }
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(ptx::smem_u32(const_cast<uint32_t *>(tmem_base_ptr)), TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_base_ptr;
  // launched as a programmatic dependent of the kernel before it in the
  // stream (the conv's staging pass, the previous GEMM): the set-up above ran
  // beside that kernel's last CTAs; global memory is touched only from here,
  // once its writes are visible
  wait_prior_grid();

  const int num_tiles = prm.tiles_m * prm.tiles_n;
  const int num_kb = prm.num_kb;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
        int mb, nb;
        gemm::tile_coords(tile, prm.tiles_m, prm.tiles_n, mb, nb, GROUP);
        const int m0 = mb * TILE_M + (int)rank * (MB * BM);  // this CTA's rows of A
        const int n0 = nb * BN + (int)rank * BN_CTA;     // this CTA's half of B
        // conv: image and first position of this CTA's rows; flat tiling
        // splits the first output pixel into (image, p, q) once per tile
        int img_a = 0, pos_a = 0, p_a = 0, q_a = 0;
        if constexpr (is_conv(EPI)) {
          img_a = mb / prm.conv_tiles_img;
          pos_a = (mb % prm.conv_tiles_img) * (2 * BM) + (int)rank * BM;
          if constexpr (EPI == Epilogue::kConv) {
            if (prm.conv_flat) {
              int f0 = mb * (2 * BM) + (int)rank * BM;  // < 2^31: checked on the host
              if (f0 >= prm.conv_n * prm.conv_pwp) f0 = 0;  // rows past the batch: any in-range start (discarded)
              img_a = f0 / prm.conv_pwp;
              pos_a = f0 - img_a * prm.conv_pwp;
              p_a = pos_a / prm.conv_wp;
              q_a = pos_a - p_a * prm.conv_wp;
            }
          }
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) { ok = false; break; }
          if (rank == 0) ptx::mbar_arrive_expect_tx(full_bar(stage), 2 * (A_STAGE_BYTES + B_STAGE_BYTES));
          const uint32_t fb = ptx::mapa(full_bar(stage), 0);
          const uint32_t a_dst = a_base + stage * A_STAGE_BYTES, b_dst = b_base + stage * B_STAGE_BYTES;
          const int k0 = kb * kblock<TI>();
          if constexpr (is_conv(EPI)) {
            const int cb = kb % prm.conv_c_blocks, rs = kb / prm.conv_c_blocks;
            const int r = rs / prm.conv_s, sx = rs % prm.conv_s;
            bool flat = false;
            if constexpr (EPI == Epilogue::kConv) flat = prm.conv_flat != 0;
            if (flat)  // 128 output pixels from (img_a, p_a, q_a) on, across rows and images, tap (r, sx)
              ptx::tma_load_im2col_4d_pair(a_dst, &tmap_a, fb, cb * gemm::BK, q_a - prm.conv_pad_w,
                                           p_a - prm.conv_pad_h, img_a, (uint16_t)sx, (uint16_t)r);
            else
              ptx::tma_load_3d_pair(a_dst, &tmap_a, fb, cb * gemm::BK,
                                    pos_a + (r - prm.conv_pad_h) * prm.conv_wp + sx, img_a);
            ptx::tma_load_3d_pair(b_dst, &tmap_b, fb, cb * gemm::BK, rs, n0);
          } else {
#pragma unroll
            for (int h = 0; h < MB; ++h) ptx::tma_load_2d_pair(a_dst + h * (BM * 128), &tmap_a, fb, k0, m0 + h * BM);
            if constexpr (B_MN_MAJOR) {
#pragma unroll
              for (int j = 0; j < BN_CTA / kblock<TI>(); ++j)
                ptx::tma_load_2d_pair(b_dst + j * (kblock<TI>() * 128), &tmap_b, fb, n0 + kblock<TI>() * j, k0);
            } else {
              ptx::tma_load_2d_pair(b_dst, &tmap_b, fb, k0, n0);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // this CTA's last loads are issued: the next kernel may be scheduled
      // (triggered earlier, a dependent's waiting CTAs sat beside the whole
      // GEMM and slowed it, e.g. the max_pool2d after a conv)
      allow_dependent_launch();
      // Wait until the MMAs have released every stage this CTA filled, so that
      // no commit arrival is still in flight towards this CTA when it exits.
      for (int i = 0; i < STAGES && ok; ++i) {
        if (!ptx::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) ok = false;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = ptx::f16_idesc(umma_format<TI>(), 0, B_MN_MAJOR ? 1 : 0, 2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs, ++local) {
        const int buf = local % NBUF;
        const uint32_t use = (uint32_t)(local / NBUF) & 1u;
        if (!ptx::mbar_wait(tempty_bar(buf), use ^ 1u, abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * MB * BN);  // A block h accumulates at + h * BN
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!ptx::mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t a_addr = a_base + stage * A_STAGE_BYTES;
          const uint32_t b_addr = b_base + stage * B_STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 4 x 32 bytes of K
            uint64_t b_desc;
            if constexpr (B_MN_MAJOR)
              b_desc = ptx::sw128_desc(b_addr + kk * mma_k<TI>() * 128, kblock<TI>() * 128, 1024);
            else
              b_desc = ptx::sw128_desc(b_addr + kk * 32, 16, 1024);
#pragma unroll
            for (int h = 0; h < MB; ++h) {
              const uint64_t a_desc = ptx::sw128_desc(a_addr + h * (BM * 128) + kk * 32, 16, 1024);
              const uint32_t d = d_tmem + (uint32_t)(h * BN);
              if constexpr (sizeof(TI) == 1)
                ptx::mma_f8_ss_pair(d, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
              else
                ptx::mma_f16_ss_pair(d, a_desc, b_desc, idesc, (kb | kk) != 0 ? 1u : 0u);
            }
          }
          ptx::mma_commit_pair_both(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) ptx::mma_commit_pair_both(tfull_bar(buf));
      }
    }
  } else if (warp < 2 + 4 * MB) {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int h = (warp - 2) >> 2;  // A block whose accumulator this warp drains
    // row-contiguous 16-byte-aligned rows: the output (and addmm's input) go
    // through the warp's shared-memory staging block
    const auto aligned16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    bool staged_epilogue = prm.son == 1 && prm.som % 8 == 0 && aligned16(prm.out);
    if constexpr (EPI == Epilogue::kAddmm)
      staged_epilogue = staged_epilogue && prm.sin == 1 && prm.sim % 8 == 0 && aligned16(prm.bias);
    (void)staged_epilogue;
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += pairs, ++local) {
      const int buf = local % NBUF;
      const uint32_t use = (uint32_t)(local / NBUF) & 1u;
      if (!ptx::mbar_wait_warp(tfull_bar(buf), use, abort_flag)) break;
      ptx::tc_fence_after();
      int mb, nb;
      gemm::tile_coords(tile, prm.tiles_m, prm.tiles_n, mb, nb, GROUP);
      if constexpr (is_conv(EPI)) {
        gemm::store_accumulator<TI, TO, EPI>(prm, tmem_base, (uint32_t)(buf * BN), quarter, lane,
                                             (int64_t)(mb % prm.conv_tiles_img) * (2 * BM) + rank * BM,
                                             (int64_t)nb * BN, mb / prm.conv_tiles_img);
      } else {
        const int64_t row0 = (int64_t)mb * TILE_M + rank * (MB * BM) + h * BM;
        bool done = false;
        if constexpr (MB == 2 && sizeof(TO) == 2) {
          if (staged_epilogue) {
            int4 *stage = reinterpret_cast<int4 *>(ctrl + CTRL_BYTES + (warp - 2) * 2048);
            gemm::store_accumulator_staged<TI, TO, EPI>(prm, tmem_base, (uint32_t)((buf * MB + h) * BN), quarter, lane,
                                                        row0, (int64_t)nb * BN, stage);
            done = true;
          }
        }
        if (!done)
          gemm::store_accumulator<TI, TO, EPI>(prm, tmem_base, (uint32_t)((buf * MB + h) * BN), quarter, lane, row0,
                                               (int64_t)nb * BN, 0);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa(tempty_bar(buf), 0));
      if constexpr (EPI == Epilogue::kConvPool)
        if (lane == 0)
          pool_count_and_push(prm, ring, mb / prm.conv_tiles_img,
                              (mb % prm.conv_tiles_img) * (2 * BM) + (int)rank * BM + quarter * 32, nb, abort_flag);
    }
    if constexpr (EPI == Epilogue::kConvPool) {
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();  // this warp's pushes are published before it counts as done
        atomicAdd(ring.epi_done, 1);
      }
    }
  } else if constexpr (EPI == Epilogue::kConvPool) {
    // ---------------------------------------------------------------- pool warps (both CTAs)
    pool_worker<TO>(prm, ring, lane, abort_flag);
  }

  __syncwarp();
  ptx::tc_fence_before();
  ptx::cluster_sync();  // no CTA leaves while its pair may still touch its shared or tensor memory
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm2

// Launches gemm_pair_kernel persistently: as many CTA pairs as can be resident
// at once (74 on a full B200), or fewer when there are fewer pair tiles.
template <typename TI, typename TO, Epilogue EPI, bool B_MN_MAJOR, int MB = 1>
int launch_pair(const CUtensorMap &ta, const CUtensorMap &tb, const gemm::Params &prm, cudaStream_t stream) {
  auto kern = gemm2::gemm_pair_kernel<TI, TO, EPI, B_MN_MAJOR, MB>;
  constexpr int threads = gemm2::threads_for(EPI, MB);
  constexpr int smem = gemm2::PairCfg<MB>::SMEM_BYTES;
  cudaError_t e = smem_optin<gemm2::gemm_pair_kernel<TI, TO, EPI, B_MN_MAJOR, MB>>(smem);
  if (e != cudaSuccess) return (int)e;
  static std::atomic<int> resident_pairs[64] = {};  // per device, filled on first use (any thread)
  int device = 0;
  cudaGetDevice(&device);
  int pairs = (device >= 0 && device < 64) ? resident_pairs[device].load(std::memory_order_relaxed) : 0;
  if (pairs == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)sm_count(), 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&pairs, kern, &cfg) != cudaSuccess || pairs <= 0) {
      cudaGetLastError();
      pairs = sm_count() / 2;
    }
    if (device >= 0 && device < 64) resident_pairs[device].store(pairs, std::memory_order_relaxed);
  }
  const int64_t tiles = (int64_t)prm.tiles_m * prm.tiles_n;
  const int grid_pairs = (int)(tiles < pairs ? tiles : pairs);
  const int launched = launch_overlapped(kern, dim3(2 * (unsigned)grid_pairs), dim3(threads), smem, stream, ta, tb, prm);
  const int st = launch_status();
  return launched != 0 ? launched : st;
}

// Launches the tensor-core GEMM when the operands meet its layout rules;
// returns kNotEligible otherwise so the caller takes the general-layout path.
template <typename TI, typename TO, Epilogue EPI>
int try_gemm(const GemmProblem &p, cudaStream_t stream) {
  if constexpr (sizeof(TI) > 2) {
    return kNotEligible;
  } else {
    using namespace gemm;
    constexpr int E = (int)sizeof(TI);
    constexpr int KB = kblock<TI>();
    if (p.K <= 0) return kNotEligible;
    if (p.M > (1LL << 31) - 1 || p.N > (1LL << 31) - 1 || p.K > (1LL << 31) - 1) return kNotEligible;
    // A must be K-contiguous with 16-byte aligned rows (TMA rules).
    const auto aligned16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    if (p.sak != 1 || (p.sam * E) % 16 != 0 || !aligned16(p.a)) return kNotEligible;
    if (p.M > 1 && p.sam < p.K) return kNotEligible;
    bool b_mn;
    if (p.sbn == 1 && (p.sbk * E) % 16 == 0 && (p.K == 1 || p.sbk >= p.N)) b_mn = true;
    else if (p.sbk == 1 && (p.sbn * E) % 16 == 0 && (p.N == 1 || p.sbn >= p.K)) b_mn = false;
    else return kNotEligible;
    if (!aligned16(p.b)) return kNotEligible;
    if (p.K * E < 16 || (b_mn && p.N * E < 16)) return kNotEligible;

    // CTA pairs (256-row tiles) unless A has a single 128-row tile
    const bool pair = p.M > BM;
    const uint32_t b_rows = pair ? (uint32_t)gemm2::BN_CTA : (uint32_t)BN;  // B rows staged per CTA
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, p.a, tmap_dtype<TI>(), E, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)p.sam, KB, BM))
      return kNotEligible;
    if (b_mn) {
      if (!make_tmap_2d(&tb, p.b, tmap_dtype<TI>(), E, (uint64_t)p.N, (uint64_t)p.K, (uint64_t)p.sbk, KB, KB))
        return kNotEligible;
    } else {
      if (!make_tmap_2d(&tb, p.b, tmap_dtype<TI>(), E, (uint64_t)p.K, (uint64_t)p.N, (uint64_t)p.sbn, KB, b_rows))
        return kNotEligible;
    }
    Params prm{};
    prm.M = p.M; prm.N = p.N; prm.K = p.K;
    prm.out = p.out; prm.som = p.som; prm.son = p.son;
    prm.bias = p.bias; prm.sim = p.sim; prm.sin = p.sin;
    prm.beta = p.beta; prm.alpha = p.alpha;
    // 512-row pair tiles (MB = 2) for 16-bit inputs when they still give
    // every CTA pair at least two tiles; 256-row ones otherwise (8-bit inputs
    // halve the MMA time per k-block, and the 4-stage ring of the 512-row
    // kernel then no longer covers the load latency)
    const int64_t tiles_n = (p.N + BN - 1) / BN;
    const bool wide = pair && E == 2 && ((p.M + 4 * BM - 1) / (4 * BM)) * tiles_n >= 2 * (sm_count() / 2);
    const int tile_m = pair ? (wide ? 4 * BM : 2 * BM) : BM;
    prm.tiles_m = (int)((p.M + tile_m - 1) / tile_m);
    prm.tiles_n = (int)tiles_n;
    prm.num_kb = (int)((p.K + KB - 1) / KB);
    const int64_t tiles = (int64_t)prm.tiles_m * prm.tiles_n;
    if (tiles > (1LL << 30)) return kNotEligible;
    if (wide)
      return b_mn ? launch_pair<TI, TO, EPI, true, 2>(ta, tb, prm, stream)
                  : launch_pair<TI, TO, EPI, false, 2>(ta, tb, prm, stream);
    if (pair)
      return b_mn ? launch_pair<TI, TO, EPI, true>(ta, tb, prm, stream)
                  : launch_pair<TI, TO, EPI, false>(ta, tb, prm, stream);
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    auto kern = b_mn ? gemm_kernel<TI, TO, EPI, true> : gemm_kernel<TI, TO, EPI, false>;
    cudaError_t e = b_mn ? smem_optin<gemm_kernel<TI, TO, EPI, true>>(SMEM_BYTES)
                         : smem_optin<gemm_kernel<TI, TO, EPI, false>>(SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    kern<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, prm);
    return launch_status();
  }
}

// ------------------------------------------------------------------ conv2d staging
// The staged input is NHWC with pad_w zero columns on each side of every row
// (row width Wp = W + 2 pad_w): pixel (h, w) of image n sits at row
// (n * H + h) * Wp + w + pad_w of a [n * H * Wp, C] matrix.  The im2col-mode
// path (flat tiling) stages without the padding columns (Wp = W, pad_w = 0):
// its TMA reads the padding as zeros from outside the tensor.

// Zeroes the pad_w columns on both sides of the staged rows whose first pixel
// lies in this CTA's pixel range [p0, p0 + 64), for channels [c0, c0 + 64):
// every row is zeroed by exactly one CTA per channel block.  C is a multiple
// of 8, so 16-byte stores.
template <typename T>
__device__ __forceinline__ void zero_pad_columns(T *dst, int p0, int HW, int W, int wp, int pad_w, int c0, int C,
                                                 int t) {
  if (pad_w == 0) return;
  const int end = p0 + 64 < HW ? p0 + 64 : HW;
  const int h_first = (p0 + W - 1) / W, h_last = (end - 1) / W;
  const int per_row = 2 * pad_w * 8;  // columns x 8 vectors of 8 channels
  for (int j = t; j < (h_last - h_first + 1) * per_row; j += 256) {
    const int h = h_first + j / per_row, rem = j % per_row, col = rem / 8, c = c0 + (rem % 8) * 8;
    const int qp = col < pad_w ? col : W + col;  // right side: W + pad_w + (col - pad_w)
    if (c < C) *reinterpret_cast<int4 *>(dst + ((int64_t)h * wp + qp) * C + c) = make_int4(0, 0, 0, 0);
  }
}

// KCRS filter (any strides) -> dense KRSC.  Done by the first z-plane of the
// input-staging grid (scheduled first), so it runs alongside the memory-bound
// input transpose instead of as a launch of its own: CTA `block` of `blocks`
// handles output channels k = block, block + blocks, ...
template <typename T>
struct FilterStaging {
  const T *in;
  T *out;
  int K, C, R, S;
  int64_t sk, sc, sr, ss;
};

template <typename T>
__device__ __forceinline__ void stage_filter(const FilterStaging<T> &f, int block, int blocks) {
  const int RS = f.R * f.S, total = RS * f.C;
  for (int k = block; k < f.K; k += blocks) {
    const T *src = f.in + (int64_t)k * f.sk;
    T *dst = f.out + (int64_t)k * total;
#pragma unroll 4
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int rs = i / f.C, c = i % f.C;
      dst[i] = src[(int64_t)c * f.sc + (int64_t)(rs / f.S) * f.sr + (int64_t)(rs % f.S) * f.ss];
    }
  }
}

// NCHW (any strides) -> W-padded NHWC, one 64-channel x 64-pixel tile per CTA
// through shared memory, so both the reads (along pixels) and the writes
// (along channels) are contiguous runs.
template <typename T>
__global__ void __launch_bounds__(256)
nchw_to_nhwc_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int HW, int W, int wp, int pad_w,
                    int64_t isn, int64_t isc, int64_t ish, int64_t isw, FilterStaging<T> filter) {
  allow_dependent_launch();  // the conv GEMM waits for this grid's writes
  if (blockIdx.z == 0) {
    stage_filter(filter, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    return;
  }
  __shared__ T tile[64][64 + 2];
  const int n = blockIdx.z - 1, c0 = blockIdx.y * 64, p0 = blockIdx.x * 64;
  const int t = threadIdx.x;
  const T *src = in + (int64_t)n * isn;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int cc = t / 64 + 4 * i, pp = t % 64;
    const int c = c0 + cc, pix = p0 + pp;
    if (c < C && pix < HW) tile[cc][pp] = src[(int64_t)c * isc + (int64_t)(pix / W) * ish + (int64_t)(pix % W) * isw];
  }
  __syncthreads();
  T *dst = out + (int64_t)n * (HW / W) * wp * C;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int pp = t / 64 + 4 * i, cc = t % 64;
    const int c = c0 + cc, pix = p0 + pp;
    if (c < C && pix < HW) dst[((int64_t)(pix / W) * wp + pix % W + pad_w) * C + c] = tile[cc][pp];
  }
  zero_pad_columns(dst, p0, HW, W, wp, pad_w, c0, C, t);
}

// Contiguous-plane NCHW -> W-padded NHWC (each (n, c) plane dense, HW a
// multiple of 8, 16-byte aligned planes, C a multiple of 8): a 64-channel x
// 64-pixel tile per CTA.  Each thread loads 8 pixels of two adjacent channels
// (16 bytes each), interleaves them into channel pairs and writes 8 words of a
// [pixel][channel] tile in shared memory; then 8 lanes store each pixel's 64
// channels as one contiguous 128-byte run.  The tile's 16-byte chunks are
// XOR-swizzled by (pixel / 8) so that both passes are free of bank conflicts.
template <typename T>
__global__ void __launch_bounds__(256)
nchw_to_nhwc_vec_kernel(const T *__restrict__ in, T *__restrict__ out, int C, int HW, int W, int wp, int pad_w,
                        int64_t isn, int64_t isc, FilterStaging<T> filter) {
  static_assert(sizeof(T) == 2, "16-bit elements");
  allow_dependent_launch();  // the conv GEMM waits for this grid's writes
  if (blockIdx.z == 0) {
    stage_filter(filter, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    return;
  }
  __shared__ __align__(16) uint32_t tile[64][32];  // [pixel][channel pair]
  const int n = blockIdx.z - 1, c0 = blockIdx.y * 64, p0 = blockIdx.x * 64;
  const int t = threadIdx.x;
  {
    const int cp = t / 8, pv = t % 8;  // channel pair 0..31, pixel group 0..7
    const int c = c0 + 2 * cp, pix = p0 + pv * 8;
    const T *src = in + (int64_t)n * isn + (int64_t)c * isc + pix;
    int4 a = make_int4(0, 0, 0, 0), b = make_int4(0, 0, 0, 0);
    if (pix < HW && c < C) {  // C % 8 == 0, so channel c + 1 exists too
      a = __ldcs(reinterpret_cast<const int4 *>(src));
      b = __ldcs(reinterpret_cast<const int4 *>(src + isc));
    }
    const uint32_t wa[4] = {(uint32_t)a.x, (uint32_t)a.y, (uint32_t)a.z, (uint32_t)a.w};
    const uint32_t wb[4] = {(uint32_t)b.x, (uint32_t)b.y, (uint32_t)b.z, (uint32_t)b.w};
    const int word = ((cp / 4) ^ pv) * 4 + cp % 4;  // rows pv * 8 + e all have row / 8 == pv
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // word j of a load holds pixels 2j (low half) and 2j + 1
      tile[pv * 8 + 2 * j][word] = __byte_perm(wa[j], wb[j], 0x5410);
      tile[pv * 8 + 2 * j + 1][word] = __byte_perm(wa[j], wb[j], 0x7632);
    }
  }
  __syncthreads();
  T *dst = out + (int64_t)n * (HW / W) * wp * C;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int v = t + 256 * i;
    const int pp = v / 8, cv = v % 8;  // pixel 0..63, vector of 8 channels 0..7
    const int pix = p0 + pp, c = c0 + cv * 8;
    if (pix < HW && c < C) {
      const int4 val = *reinterpret_cast<const int4 *>(&tile[pp][((cv ^ (pp / 8)) & 7) * 4]);
      const int64_t row = (int64_t)(pix / W) * wp + pix % W + pad_w;
      *reinterpret_cast<int4 *>(dst + row * C + c) = val;
    }
  }
  zero_pad_columns(dst, p0, HW, W, wp, pad_w, c0, C, t);
}

// Workspace of the tensor-core conv2d path: the W-padded NHWC input, then the
// KRSC filter at the next 256-byte boundary.  0 when the path does not apply.
inline int64_t conv_workspace_bytes(int64_t n, int64_t c, int64_t h, int64_t w, int64_t k, int64_t r, int64_t s,
                                    int64_t pad_w, int elem) {
  if (elem != 2 || c % 8 != 0) return 0;
  const int64_t act = n * h * (w + 2 * pad_w) * c * elem;
  const int64_t flt = k * r * s * c * elem;
  return ((act + 255) / 256) * 256 + flt;
}

template <typename T>
int try_conv(const ConvProblem &p, void *workspace, int64_t workspace_bytes, cudaStream_t stream,
             const PoolFusion *pool = nullptr) {
  if constexpr (sizeof(T) != 2) {
    return kNotEligible;
  } else {
    using namespace gemm;
    const int64_t need = conv_workspace_bytes(p.n, p.c, p.h, p.w, p.k, p.r, p.s, p.pad_w, 2);
    if (need == 0 || workspace == nullptr || workspace_bytes < need) return kNotEligible;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return kNotEligible;
    const int64_t wp = p.w + 2 * p.pad_w;
    // the fused pool runs in the CTA-pair kernel, one 32-position block per
    // epilogue warp spanning at most two conv rows; its work codes
    // (8 per pool row of a channel tile) must fit an int
    if (pool && (p.P * wp <= BM || wp < 32 || p.Q % 8 != 0 || p.Q > 64 || pool->os[3] != 1 || pool->os[0] % 4 != 0 ||
                 pool->os[1] % 4 != 0 || pool->os[2] % 4 != 0 || (reinterpret_cast<uintptr_t>(pool->out) & 7u) != 0 ||
                 p.n * ((p.k + BN - 1) / BN) * pool->P2 * 8 >= (1LL << 31)))
      return kNotEligible;
    if (p.h == 0 || p.w == 0 || p.n >= 65535 || p.c > (1 << 20) || p.h > (1 << 20) || wp > (1 << 20) ||
        p.k > (1 << 20) || p.r * p.s * p.c > (1 << 30) || p.pad_h > (1 << 20) ||
        (p.h + 2 * p.pad_h + p.r) * wp > (1LL << 30))
      return kNotEligible;
    // CTA pairs (256-position tiles) unless an image has a single 128-position tile
    const bool pair = p.P * wp > BM;
    const int tile_m = pair ? 2 * BM : BM;
    // Flat tiling for the CTA-pair conv without the fused pool: the batch's
    // N * P * Q output pixels are one range of tiles, whose A rows
    // im2col-mode TMA walks across rows and images of the unpadded NHWC input
    // (padding read as zeros from outside the tensor).  The map's box corners
    // (-pad, pad - (filter - 1)) must lie in [-128, 127]; inputs under 128 KB
    // keep the padded-row path.
    const bool flat = pair && !pool && p.pad_h <= 127 && p.pad_w <= 127 && p.r - 1 - p.pad_h <= 128 &&
                      p.s - 1 - p.pad_w <= 128 && p.r <= 255 && p.s <= 255 && p.n * p.h * p.w * p.c * 2 >= 131072 &&
                      p.n * p.P * p.Q < (1LL << 31) - 2 * tile_m && encode_im2col_fn() != nullptr;
    const int64_t wp_stage = flat ? p.w : wp, pad_w_stage = flat ? 0 : p.pad_w;
    // a dense channels-last (NHWC) input is already what the im2col map
    // reads: only the filter is staged
    const bool nhwc_input = flat && p.is[1] == 1 && p.is[3] == p.c && p.is[2] == p.w * p.c &&
                            p.is[0] == p.h * p.w * p.c && (reinterpret_cast<uintptr_t>(p.input) & 15u) == 0;
    T *act = nhwc_input ? const_cast<T *>(static_cast<const T *>(p.input)) : static_cast<T *>(workspace);
    T *flt = reinterpret_cast<T *>(static_cast<uint8_t *>(workspace) + ((p.n * p.h * wp * p.c * 2 + 255) / 256) * 256);
    {
      const int HW = (int)(p.h * p.w);
      // z-plane 0: the filter; planes 1 .. n: the images
      dim3 grid((unsigned)((HW + 63) / 64), (unsigned)((p.c + 63) / 64), (unsigned)(nhwc_input ? 1 : p.n + 1));
      const FilterStaging<T> filter{static_cast<const T *>(p.filter), flt, (int)p.k, (int)p.c, (int)p.r, (int)p.s,
                                    p.fs[0], p.fs[1], p.fs[2], p.fs[3]};
      const bool dense_planes = p.is[3] == 1 && p.is[2] == p.w && HW % 8 == 0 && p.is[1] % 8 == 0 &&
                                p.is[0] % 8 == 0 && (reinterpret_cast<uintptr_t>(p.input) & 15u) == 0;
      if (dense_planes)
        nchw_to_nhwc_vec_kernel<T><<<grid, 256, 0, stream>>>(static_cast<const T *>(p.input), act, (int)p.c, HW,
                                                             (int)p.w, (int)wp_stage, (int)pad_w_stage, p.is[0],
                                                             p.is[1], filter);
      else
        nchw_to_nhwc_kernel<T><<<grid, 256, 0, stream>>>(static_cast<const T *>(p.input), act, (int)p.c, HW,
                                                         (int)p.w, (int)wp_stage, (int)pad_w_stage, p.is[0],
                                                         p.is[1], p.is[2], p.is[3], filter);
      const int st = launch_status();
      if (st != 0) return st;
    }
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return kNotEligible;
    CUtensorMap ta, tb;
    if (flat) {
      // NHWC dims {C, W, H, N}; the box walks output pixels: corners {W, H}
      const cuuint64_t dims[4] = {(cuuint64_t)p.c, (cuuint64_t)p.w, (cuuint64_t)p.h, (cuuint64_t)p.n};
      const cuuint64_t strides[3] = {(cuuint64_t)(p.c * 2), (cuuint64_t)(p.w * p.c * 2),
                                     (cuuint64_t)(p.h * p.w * p.c * 2)};
      const int lower[2] = {-(int)p.pad_w, -(int)p.pad_h};
      const int upper[2] = {(int)(p.pad_w - (p.s - 1)), (int)(p.pad_h - (p.r - 1))};
      const cuuint32_t estr[4] = {1, 1, 1, 1};
      if (encode_im2col_fn()(&ta, tmap_dtype<T>(), 4, act, dims, strides, lower, upper, 64, (cuuint32_t)BM, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return kNotEligible;
    } else {
      // [image][H * Wp rows][C]: one image per outer index, so rows shifted
      // above or below an image read as zero instead of a neighbour's pixels
      const cuuint64_t dims[3] = {(cuuint64_t)p.c, (cuuint64_t)(p.h * wp), (cuuint64_t)p.n};
      const cuuint64_t strides[2] = {(cuuint64_t)(p.c * 2), (cuuint64_t)(p.h * wp * p.c * 2)};
      const cuuint32_t box[3] = {64, (cuuint32_t)BM, 1};
      const cuuint32_t estr[3] = {1, 1, 1};
      if (fn(&ta, tmap_dtype<T>(), 3, act, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return kNotEligible;
    }
    {
      const cuuint64_t dims[3] = {(cuuint64_t)p.c, (cuuint64_t)(p.r * p.s), (cuuint64_t)p.k};
      const cuuint64_t strides[2] = {(cuuint64_t)(p.c * 2), (cuuint64_t)(p.r * p.s * p.c * 2)};
      const cuuint32_t box[3] = {64, 1, (cuuint32_t)(pair ? gemm2::BN_CTA : BN)};
      const cuuint32_t estr[3] = {1, 1, 1};
      if (fn(&tb, tmap_dtype<T>(), 3, flt, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return kNotEligible;
    }
    Params prm{};
    prm.out = p.output;
    prm.conv_c_blocks = (int)((p.c + BK - 1) / BK);
    prm.conv_s = (int)p.s;
    prm.conv_pad_h = (int)p.pad_h;
    prm.conv_wp = (int)wp;
    prm.conv_tiles_img = (int)((p.P * wp + tile_m - 1) / tile_m);
    prm.conv_P = (int)p.P;
    prm.conv_Q = (int)p.Q;
    prm.conv_osn = p.os[0];
    prm.conv_osk = p.os[1];
    prm.conv_osp = p.os[2];
    prm.conv_osq = p.os[3];
    prm.conv_n = (int)p.n;
    prm.conv_pad_w = (int)p.pad_w;
    if (flat) {
      prm.conv_flat = 1;
      prm.conv_wp = (int)p.Q;  // no padding columns
      prm.conv_pwp = (int)(p.P * p.Q);
      prm.conv_tiles_img = (int)((p.n * p.P * p.Q + tile_m - 1) / tile_m);  // all tiles in one range
    }
    const int64_t tiles_m = flat ? prm.conv_tiles_img : p.n * prm.conv_tiles_img;
    prm.tiles_m = (int)tiles_m;
    prm.tiles_n = (int)((p.k + BN - 1) / BN);
    prm.num_kb = (int)(p.r * p.s * prm.conv_c_blocks);
    prm.M = tiles_m * tile_m;
    prm.N = p.k;
    prm.K = p.r * p.s * p.c;
    const int64_t tiles = tiles_m * prm.tiles_n;
    if (tiles > (1LL << 30)) return kNotEligible;
    if (pool) {
      prm.pool_out = pool->out;
      prm.pool_osn = pool->os[0];
      prm.pool_osk = pool->os[1];
      prm.pool_osi = pool->os[2];
      prm.pool_osj = pool->os[3];
      prm.pool_P = pool->P2;
      prm.pool_Q = pool->Q2;
      prm.pool_counters = pool->counters;
      const cudaError_t e = cudaMemsetAsync(pool->counters, 0, (size_t)p.n * prm.tiles_n * pool->P2 * sizeof(int),
                                            stream);
      if (e != cudaSuccess) return (int)e;
      return launch_pair<T, T, Epilogue::kConvPool, false>(ta, tb, prm, stream);
    }
    if (pair) return launch_pair<T, T, Epilogue::kConv, false>(ta, tb, prm, stream);
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    auto kern = gemm_kernel<T, T, Epilogue::kConv, false>;
    cudaError_t e = smem_optin<gemm_kernel<T, T, Epilogue::kConv, false>>(SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    kern<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, prm);
    return launch_status();
  }
}

}  // namespace tc
}  // namespace nt
