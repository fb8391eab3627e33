// tcgen05 flash attention for the reference's exp-reduction-dot-region program
// (tests/test_attention.py:14-70), with the application's numerics:
//   q' = round(q * round(log2 e))            (in the input dtype)
//   s  = q' k^T                              (fp32, tensor cores)
//   keys >= seq_kv and (causal) keys > query masked to -inf
//   m_new = max(m, rowmax s); p = exp2(s - m_new); alpha = exp2(m - m_new)
//   o = o * alpha + round(p) v; l = l * alpha + rowsum p   (m = -inf, l = 1 at start)
//   out = round(o / l)
//
// Persistent: one CTA per SM loops over work items (batch, head, 256 queries)
// = two 128-row Q tiles; 10 warps:
//   warp 0     TMA producer: an item's two Q tiles (each once the previous
//              item's last QK of that tile has read it), then K_j and V_j
//              (128 keys each) through a 5-slot shared-memory ring that runs
//              on across items;
//   warp 1     allocates TMEM and issues the MMAs from one thread, tile by
//              tile: S_t = Q_t K_j^T into tile t's S columns, then
//              O_t += P_t V_j with P_t read from tensor memory;
//   warps 2-5, 6-9  one warpgroup per Q tile, one thread per query row (= TMEM
//              lane): scale Q in place, read S from TMEM, online softmax in
//              registers, rescale O in TMEM when the row max moved far enough,
//              write P (rounded to the input dtype, two per 32-bit column)
//              over S's columns, and finally read O out of TMEM (releasing it
//              to the next item) and store O / l to global memory.
// While one tile's softmax runs, the tensor cores work on the other tile; an
// item's epilogue and the next item's Q load overlap the other tile's work.
// Items are dealt out head by head in alternating-direction rounds (causal:
// longest first within a round); causal items skip key blocks above the
// diagonal.  Every mbarrier wait is bounded in time.
#pragma once

#include <cuda.h>
#include "common.cuh"
#include "ptx.cuh"
#include "gemm_tc.cuh"

namespace nt {
namespace tc {

struct AttentionProblem {
  const void *q, *k, *v;
  void *o;
  int64_t B, H, SQ, SK, D;
  int64_t qsb, qsh, qss, qsd, ksb, ksh, kss, ksd, vsb, vsh, vss, vsd, osb, osh, oss, osd;
  bool causal;
  float log2e;
};

namespace attn {

constexpr int BM = 128;     // queries per Q tile
constexpr int BN = 128;     // keys per block
constexpr int TILES = 2;    // Q tiles per CTA, one softmax warpgroup each
constexpr int RING = 5;     // K/V shared-memory slots (K_j, V_j, K_j+1, ... in load order)
constexpr int THREADS = 64 + TILES * 128;
static_assert(TILES == 2, "the MMA issuer interleaves exactly two Q tiles");
constexpr int TMEM_COLS = 512;
// A row's running max is only moved when a block's max exceeds it by more
// than 2^kRescaleLog2<T> (log2 domain); otherwise p = exp2(s - m) is taken
// against the stale max, so p <= 2^kRescaleLog2 -- within float16's range
// (2^14 < 65504) and far inside bfloat16's.  o / l is unchanged mathematically,
// the relative precision of p is the same at any scale, and O is rescaled in
// TMEM only on the rare large jumps.
template <typename T> struct RescaleLog2;
template <> struct RescaleLog2<__half> { static constexpr float value = 14.f; };
template <> struct RescaleLog2<__nv_bfloat16> { static constexpr float value = 24.f; };

template <int DP>  // head_dim padded to 64 or 128
struct Layout {
  static constexpr int ATOMS = DP / 64;                // 128-byte swizzle atoms along head_dim
  static constexpr int Q_BYTES = BM * DP * 2;          // one Q tile
  static constexpr int KV_BYTES = BN * DP * 2;         // one K or V block
  static constexpr int Q_OFF = 0;
  static constexpr int RING_OFF = Q_OFF + TILES * Q_BYTES;
  static constexpr int CTRL_OFF = RING_OFF + RING * KV_BYTES;
  static constexpr int SMEM_BYTES = CTRL_OFF + 256 + 1024;
  static_assert(112 + 16 * RING <= 240, "barrier slots");
};

struct Params {
  int B, H, SQ, SK, D;
  int q_pairs;  // CTAs per (batch, head): ceil(SQ / (TILES * BM))
  int causal;
  float log2e;
  void *o;
  int64_t osb, osh, oss, osd;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

template <typename T, int DP>
__global__ void __launch_bounds__(THREADS, 1)
attention_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                 const __grid_constant__ CUtensorMap tmap_v, Params prm) {
  using L = Layout<DP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  const uint32_t ctrl = base + L::CTRL_OFF;
  // barrier slots (8 bytes each), per Q tile t unless noted
  auto q_full = [&](int t) { return ctrl + 8u * t; };         // Q_t landed (TMA)
  auto q_ready = [&](int t) { return ctrl + 16 + 8u * t; };   // Q_t scaled by its softmax warps
  auto q_free = [&](int t) { return ctrl + 32 + 8u * t; };    // last QK_t of the work item done
  auto s_full = [&](int t) { return ctrl + 48 + 8u * t; };    // S_t of a key block in TMEM
  auto p_full = [&](int t) { return ctrl + 64 + 8u * t; };    // P_t written (and O_t rescaled)
  auto o_done = [&](int t) { return ctrl + 80 + 8u * t; };    // last PV_t of the work item done
  auto o_free = [&](int t) { return ctrl + 96 + 8u * t; };    // O_t read out by the epilogue
  auto slot_full = [&](int s) { return ctrl + 112 + 8u * s; };
  auto slot_empty = [&](int s) { return ctrl + 112 + 8u * RING + 8u * s; };
  volatile uint32_t *tmem_base_ptr = reinterpret_cast<volatile uint32_t *>(smem + L::CTRL_OFF + 240);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::CTRL_OFF + 244);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_head = prm.q_pairs;
  const int heads = prm.B * prm.H;
  const int num_items = heads * per_head;
  const int kv_blocks = (prm.SK + BN - 1) / BN;

  // Work item k = (batch, head, pair of Q tiles), head-major: k = bh *
  // per_head + pair.  Items are dealt in rounds of G = gridDim.x consecutive
  // items (about G / per_head heads, whose K and V then stay in L2 while the
  // round's CTAs stream them), alternating the direction each round (CTA c
  // takes the round's c-th item, then its (G-1-c)-th).  Causal items differ in
  // length, so within a round they are taken longest pair first: with the
  // alternating direction every CTA's share of the work comes out nearly equal.
  struct Item {
    int b, h, q0;
  };
  auto item = [&](int k) {
    const int bh = k / per_head, qp = k % per_head;
    return Item{bh / prm.H, bh % prm.H, qp * (TILES * BM)};
  };
  // p-th item of round w in order of decreasing pair index (ties by k).
  auto round_item = [&](int w, int p) {
    const int lo = w * (int)gridDim.x;
    const int hi = min(lo + (int)gridDim.x, num_items);
    if (!prm.causal) return lo + p;
    for (int v = per_head - 1; v >= 0; --v) {
      const int first = lo + ((v - lo) % per_head + per_head) % per_head;  // first k >= lo with k % per_head == v
      const int count = first >= hi ? 0 : (hi - 1 - first) / per_head + 1;
      if (p < count) return first + p * per_head;
      p -= count;
    }
    return -1;
  };
  // The CTA's i-th item, or -1 when it has none left.
  auto nth_item = [&](int i) {
    const int g = (int)gridDim.x, c = (int)blockIdx.x;
    if ((int64_t)i * g >= num_items) return -1;
    const int size = min(g, num_items - i * g);
    const int p = (i & 1) ? g - 1 - c : c;
    return p < size ? round_item(i, p) : -1;
  };
  // key blocks Q tile t of an item starting at query q0 needs (causal: up to
  // its diagonal block)
  auto n_blk = [&](int q0, int t) {
    return prm.causal ? min(kv_blocks, (q0 + t * BM + BM - 1) / BN + 1) : kv_blocks;
  };

  if (threadIdx.x == 0) {
    for (int t = 0; t < TILES; ++t) {
      ptx::mbar_init(q_full(t), 1);
      ptx::mbar_init(q_ready(t), 128);
      ptx::mbar_init(q_free(t), 1);
      ptx::mbar_init(s_full(t), 1);
      ptx::mbar_init(p_full(t), 128);
      ptx::mbar_init(o_done(t), 1);
      ptx::mbar_init(o_free(t), 128);
    }
    for (int s = 0; s < RING; ++s) {
      ptx::mbar_init(slot_full(s), 1);
      ptx::mbar_init(slot_empty(s), 1);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tmap_q);
    ptx::prefetch_tmap(&tmap_k);
    ptx::prefetch_tmap(&tmap_v);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(const_cast<uint32_t *>(tmem_base_ptr)), TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_base_ptr;
  auto tmem_s = [&](int t) { return tmem_base + (uint32_t)(t * BN); };
  auto tmem_o = [&](int t) { return tmem_base + (uint32_t)(TILES * BN + t * 128); };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      int r = 0;  // ring items issued so far (all work items)
      for (int it = 0, k = nth_item(0); k >= 0 && ok; k = nth_item(++it)) {
        const Item w = item(k);
        const int n_max = n_blk(w.q0, TILES - 1);
        // Q_t of this item once the previous item's last QK_t has read Q_t
        for (int t = 0; t < TILES && ok; ++t) {
          if (it > 0 && !ptx::mbar_wait(q_free(t), (uint32_t)(it - 1) & 1u, abort_flag)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(q_full(t), L::Q_BYTES);
          for (int a = 0; a < L::ATOMS; ++a)
            ptx::tma_load_4d(base + L::Q_OFF + t * L::Q_BYTES + a * (BM * 128), &tmap_q, q_full(t), 64 * a,
                             w.q0 + t * BM, w.h, w.b);
        }
        // ring items in order K_0, V_0, K_1, V_1, ...
        for (int i = 0; i < 2 * n_max && ok; ++i, ++r) {
          const int slot = r % RING;
          const uint32_t use = (uint32_t)(r / RING) & 1u;
          if (!ptx::mbar_wait(slot_empty(slot), use ^ 1u, abort_flag)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(slot_full(slot), L::KV_BYTES);
          const CUtensorMap *map = (i & 1) ? &tmap_v : &tmap_k;
          for (int a = 0; a < L::ATOMS; ++a)
            ptx::tma_load_4d(base + L::RING_OFF + slot * L::KV_BYTES + a * (BN * 128), map, slot_full(slot), 64 * a,
                             (i >> 1) * BN, w.h, w.b);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = umma_format<T>();
      constexpr uint32_t idesc_qk = ptx::f16_idesc(fmt, 0, 0, BM, BN);  // B = K block, K-major
      constexpr uint32_t idesc_pv = ptx::f16_idesc(fmt, 0, 1, BM, DP);  // B = V block, MN-major
      auto slot_addr = [&](int r) { return base + L::RING_OFF + (r % RING) * L::KV_BYTES; };
      auto wait_item = [&](int r) {
        return ptx::mbar_wait(slot_full(r % RING), (uint32_t)(r / RING) & 1u, abort_flag);
      };
      auto issue_qk = [&](int t, int r) {
        const uint32_t kb = slot_addr(r);
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk) {
          const uint32_t off = (kk / 4) * (BM * 128) + (kk % 4) * 32;
          const uint32_t koff = (kk / 4) * (BN * 128) + (kk % 4) * 32;
          const uint64_t a_desc = ptx::sw128_desc(base + L::Q_OFF + t * L::Q_BYTES + off, 16, 1024);
          const uint64_t b_desc = ptx::sw128_desc(kb + koff, 16, 1024);
          ptx::mma_f16_ss(tmem_s(t), a_desc, b_desc, idesc_qk, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(s_full(t));
      };
      auto issue_pv = [&](int t, int r, bool first) {
        const uint32_t vb = slot_addr(r);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // P_t: 128 keys packed two per column in tile t's S columns
          const uint64_t b_desc = ptx::sw128_desc(vb + kk * 16 * 128, BN * 128, 1024);
          ptx::mma_f16_ts(tmem_o(t), tmem_s(t) + (uint32_t)(kk * 8), b_desc, idesc_pv, (!first || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = true;
      int r = 0;                 // ring position of this item's K_0
      int blk[TILES] = {0, 0};   // key blocks of tile t in earlier items (s_full / p_full phases)
      for (int it = 0, k = nth_item(0); k >= 0 && ok; k = nth_item(++it)) {
        const Item w = item(k);
        const int n0 = n_blk(w.q0, 0), n1 = n_blk(w.q0, 1);
        const int n_max = n1;
        ok = wait_item(r);  // K_0
        for (int t = 0; t < TILES && ok; ++t) {
          if (!ptx::mbar_wait(q_ready(t), (uint32_t)it & 1u, abort_flag)) { ok = false; break; }
          ptx::tc_fence_after();
          issue_qk(t, r);
          if ((t == 0 ? n0 : n1) == 1) ptx::mma_commit(q_free(t));
        }
        if (!ok) break;
        ptx::mma_commit(slot_empty(r % RING));  // K_0 read by every tile's first QK
        for (int j = 0; j < n_max && ok; ++j) {
          const int rv = r + 2 * j + 1, rk = r + 2 * j + 2;
          if (!wait_item(rv)) { ok = false; break; }  // V_j
          bool k_next_waited = false;
          for (int t = 0; t < TILES && ok; ++t) {
            const int n_t = t == 0 ? n0 : n1;
            if (j >= n_t) continue;
            // P_t(j) ready also means the softmax has read S_t(j), so S_t may be
            // overwritten by the next QK of this tile.
            if (!ptx::mbar_wait(p_full(t), (uint32_t)(blk[t] + j) & 1u, abort_flag)) { ok = false; break; }
            // the first PV of an item overwrites O_t: the previous item's
            // epilogue must have read it
            if (j == 0 && it > 0 && !ptx::mbar_wait(o_free(t), (uint32_t)(it - 1) & 1u, abort_flag)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            issue_pv(t, rv, j == 0);
            // O_t is read by the softmax warps only after the last block
            if (j == n_t - 1) ptx::mma_commit(o_done(t));
            if (j + 1 < n_t) {
              if (!k_next_waited) {
                if (!wait_item(rk)) { ok = false; break; }
                k_next_waited = true;
                ptx::tc_fence_after();
              }
              issue_qk(t, rk);
              if (j + 2 == n_t) ptx::mma_commit(q_free(t));  // that was tile t's last QK
            }
          }
          if (!ok) break;
          ptx::mma_commit(slot_empty(rv % RING));                  // V_j
          if (k_next_waited) ptx::mma_commit(slot_empty(rk % RING));  // K_j+1
        }
        r += 2 * n_max;
        blk[0] += n0;
        blk[1] += n1;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax / correction / epilogue
    const int t = (warp - 2) / 4;  // Q tile of this warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    int blk = 0;  // key blocks of this tile in earlier items
    for (int it = 0, k = nth_item(0); k >= 0 && ok; k = nth_item(++it)) {
      const Item w = item(k);
      const int qi = w.q0 + t * BM + row;
      const int n_t = n_blk(w.q0, t);
      ok = ptx::mbar_wait_warp(q_full(t), (uint32_t)it & 1u, abort_flag);
      if (ok) {
        // q' = round(q * round(log2 e)) in place; a thread owns its row's
        // 128-byte segment in every atom, so the swizzle does not matter.  It
        // walks the segment's eight 16-byte chunks starting at chunk row % 8,
        // so that the 8 lanes of a shared-memory phase touch 8 different
        // chunks of 8 rows (all 32 banks) instead of one chunk column (an
        // 8-way conflict that made this step take about 4 us per item).
#pragma unroll
        for (int a = 0; a < L::ATOMS; ++a) {
          int4 *seg = reinterpret_cast<int4 *>(smem + L::Q_OFF + t * L::Q_BYTES + a * (BM * 128) + row * 128);
#pragma unroll 2
          for (int c = 0; c < 8; ++c) {
            const int cc = (c + row) & 7;
            int4 raw = seg[cc];
            T *e = reinterpret_cast<T *>(&raw);
#pragma unroll
            for (int i = 0; i < 8; ++i) e[i] = from_f<T>(to_f(e[i]) * prm.log2e);
            seg[cc] = raw;
          }
        }
        ptx::fence_proxy_async_smem();
      }
      ptx::mbar_arrive(q_ready(t));
      if (!ok) break;

      float m_i = -INFINITY, l_i = 1.f;
      for (int j = 0; j < n_t && ok; ++j) {
        if (!ptx::mbar_wait_warp(s_full(t), (uint32_t)(blk + j) & 1u, abort_flag)) { ok = false; break; }
        ptx::tc_fence_after();
        uint32_t sr[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          ptx::tmem_ld_32x32b_x32(tmem_s(t) + lane_base + (uint32_t)(c * 32),
                                  *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
        ptx::tmem_ld_wait();
        float *sv = reinterpret_cast<float *>(sr);
        if (j == n_t - 1) {
          // the last block of a tile holds the key tail and (causal) the diagonal
          const int k0 = j * BN;
          int limit = prm.SK - k0;
          if (prm.causal) limit = min(limit, qi - k0 + 1);
#pragma unroll
          for (int c = 0; c < BN; ++c) sv[c] = c < limit ? sv[c] : -INFINITY;
        }
        // 8 independent partial maxima/sums keep the reductions off one long
        // dependency chain.
        float mp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mp[u] = sv[u];
#pragma unroll
        for (int c = 8; c < BN; ++c) mp[c & 7] = fmaxf(mp[c & 7], sv[c]);
#pragma unroll
        for (int u = 4; u > 0; u >>= 1)
#pragma unroll
          for (int v = 0; v < u; ++v) mp[v] = fmaxf(mp[v], mp[v + u]);
        const float m_blk = mp[0];
        const bool move = m_blk > m_i + RescaleLog2<T>::value;  // true on the first block (m_i = -inf)
        const float m_new = move ? m_blk : m_i;
        const float alpha = move ? ex2(m_i - m_new) : 1.f;
        // p = exp2(s - m) in two halves of 64 keys; each half is packed (two keys
        // per 32-bit column) and stored over this tile's S columns as soon as it
        // is done, so the first store's latency overlaps the second half's
        // exponentials.  Column c holds keys 2c (low half) and 2c + 1: the
        // A-operand layout of the PV MMA.
        float lp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int h2 = 0; h2 < BN / 64; ++h2) {
          uint32_t packed[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int c = h2 * 64 + 2 * i;
            const float p0 = ex2(sv[c] - m_new), p1 = ex2(sv[c + 1] - m_new);
            lp[(2 * i) & 7] += p0;
            lp[(2 * i + 1) & 7] += p1;
            packed[i] = pack2<T>(p0, p1);
          }
          ptx::tmem_st_32x32b_x32(tmem_s(t) + lane_base + (uint32_t)(h2 * 32), packed);
        }
#pragma unroll
        for (int u = 4; u > 0; u >>= 1)
#pragma unroll
          for (int v = 0; v < u; ++v) lp[v] += lp[v + u];
        const float l_blk = lp[0];
        // O_t holds P(j-1) V(j-1) already: the commit that signalled S_t(j) came
        // after that MMA, and a commit covers every earlier MMA of its thread.
        // The rescale reuses the registers S held; it must land before the PV MMA
        // of this block, which waits for p_full below.
        if (j > 0 && __any_sync(0xffffffffu, move)) {
          uint32_t orow[DP];
#pragma unroll
          for (int c = 0; c < DP / 32; ++c)
            ptx::tmem_ld_32x32b_x32(tmem_o(t) + lane_base + (uint32_t)(c * 32),
                                    *reinterpret_cast<uint32_t(*)[32]>(&orow[c * 32]));
          ptx::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < DP; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
#pragma unroll
          for (int c = 0; c < DP / 32; ++c)
            ptx::tmem_st_32x32b_x32(tmem_o(t) + lane_base + (uint32_t)(c * 32),
                                    *reinterpret_cast<uint32_t(*)[32]>(&orow[c * 32]));
        }
        m_i = m_new;
        l_i = l_i * alpha + l_blk;
        ptx::tmem_st_wait();
        ptx::tc_fence_before();
        ptx::mbar_arrive(p_full(t));
      }
      if (!ok) break;
      blk += n_t;

      // epilogue: O_t is read out of TMEM first and released (the next item's
      // first PV_t may then overwrite it), then O / l goes to global memory.
      if (!ptx::mbar_wait_warp(o_done(t), (uint32_t)it & 1u, abort_flag)) { ok = false; break; }
      ptx::tc_fence_after();
      uint32_t orow[DP];
#pragma unroll
      for (int c = 0; c < DP / 32; ++c)
        ptx::tmem_ld_32x32b_x32(tmem_o(t) + lane_base + (uint32_t)(c * 32),
                                *reinterpret_cast<uint32_t(*)[32]>(&orow[c * 32]));
      ptx::tmem_ld_wait();
      ptx::tc_fence_before();
      ptx::mbar_arrive(o_free(t));
      const float inv = 1.f / l_i;
      T *out = static_cast<T *>(prm.o) + (int64_t)w.b * prm.osb + (int64_t)w.h * prm.osh + (int64_t)qi * prm.oss;
      if (qi < prm.SQ) {
        if (prm.D == DP && prm.osd == 1 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
#pragma unroll
          for (int v8 = 0; v8 < DP / 8; ++v8) {
            const float *o8 = reinterpret_cast<const float *>(orow + v8 * 8);
            const int4 pk = make_int4((int)pack2<T>(o8[0] * inv, o8[1] * inv), (int)pack2<T>(o8[2] * inv, o8[3] * inv),
                                      (int)pack2<T>(o8[4] * inv, o8[5] * inv), (int)pack2<T>(o8[6] * inv, o8[7] * inv));
            *reinterpret_cast<int4 *>(out + v8 * 8) = pk;
          }
        } else {
#pragma unroll
          for (int i = 0; i < DP; ++i)
            if (i < prm.D) out[(int64_t)i * prm.osd] = from_f<T>(__uint_as_float(orow[i]) * inv);
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// 4-D tensor map over a [batch, heads, seq, head_dim] tensor with unit
// head_dim stride: dims (head_dim, seq, heads, batch), box (64, 128, 1, 1),
// 128-byte swizzle; rows past seq and columns past head_dim read as zero.
inline bool make_tmap_bhsd(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int64_t B, int64_t H,
                           int64_t S, int64_t D, int64_t sb, int64_t sh, int64_t ss) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, 128, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, dt, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace attn

template <typename T>
int try_attention(const AttentionProblem &p, cudaStream_t stream) {
  if constexpr (sizeof(T) != 2) {
    return kNotEligible;
  } else {
    using namespace attn;
    if (p.D <= 0 || p.D > 128 || p.SK <= 0 || p.SQ <= 0) return kNotEligible;
    const auto aligned16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
    if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v)) return kNotEligible;
    if (p.qsd != 1 || p.ksd != 1 || p.vsd != 1) return kNotEligible;
    for (int64_t st : {p.qsb, p.qsh, p.qss, p.ksb, p.ksh, p.kss, p.vsb, p.vsh, p.vss})
      if ((st * 2) % 16 != 0 || st <= 0) return kNotEligible;
    if (p.B > 65535 || p.H > 65535 || p.SQ > (1 << 30) || p.SK > (1 << 30)) return kNotEligible;
    CUtensorMap tq, tk, tv;
    const CUtensorMapDataType dt = tmap_dtype<T>();
    if (!make_tmap_bhsd(&tq, p.q, dt, p.B, p.H, p.SQ, p.D, p.qsb, p.qsh, p.qss) ||
        !make_tmap_bhsd(&tk, p.k, dt, p.B, p.H, p.SK, p.D, p.ksb, p.ksh, p.kss) ||
        !make_tmap_bhsd(&tv, p.v, dt, p.B, p.H, p.SK, p.D, p.vsb, p.vsh, p.vss))
      return kNotEligible;
    Params prm;
    prm.B = (int)p.B; prm.H = (int)p.H; prm.SQ = (int)p.SQ; prm.SK = (int)p.SK; prm.D = (int)p.D;
    prm.q_pairs = (int)((p.SQ + TILES * BM - 1) / (TILES * BM));
    prm.causal = p.causal ? 1 : 0;
    prm.log2e = p.log2e;
    prm.o = p.o;
    prm.osb = p.osb; prm.osh = p.osh; prm.oss = p.oss; prm.osd = p.osd;
    const int64_t items = p.B * p.H * prm.q_pairs;
    if (items > (1LL << 31) - 1) return kNotEligible;
    const int64_t grid = items < sm_count() ? items : sm_count();  // persistent: one CTA per SM
    if (p.D <= 64) {
      auto kern = attention_kernel<T, 64>;
      cudaError_t e = smem_optin<attention_kernel<T, 64>>(Layout<64>::SMEM_BYTES);
      if (e != cudaSuccess) return (int)e;
      kern<<<(unsigned)grid, THREADS, Layout<64>::SMEM_BYTES, stream>>>(tq, tk, tv, prm);
    } else {
      auto kern = attention_kernel<T, 128>;
      cudaError_t e = smem_optin<attention_kernel<T, 128>>(Layout<128>::SMEM_BYTES);
      if (e != cudaSuccess) return (int)e;
      kern<<<(unsigned)grid, THREADS, Layout<128>::SMEM_BYTES, stream>>>(tq, tk, tv, prm);
    }
    return launch_status();
  }
}

}  // namespace tc
}  // namespace nt
