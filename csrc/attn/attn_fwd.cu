// Causal / full flash-attention forward on sm_100a tensor cores (tcgen05 + TMEM).
//
// Replaces the reference's F.scaled_dot_product_attention call and its GQA
// expansion (tinytron/model/modules/attn.py:66-83, 420-423): K/V heads are never
// repeated — q head h reads kv head h / (Hq/Hkv) directly.
//
// Layout: Q, K, V are read in place from token-major buffers (row = token,
// head h occupies columns [col0 + h*D, col0 + (h+1)*D)), which is exactly the
// packed output of the fused QKV projection, so no permute kernels run.  O is
// written token-major [tokens, Hq*D] (the c_proj input layout); LSE (natural log)
// is written [B, Hq, T] for the backward pass.
//
// One CTA = one (batch, q head, pair of 128-query tiles).  Warp roles (384 threads):
//   TMA producer: both Q tiles once; K/V tiles through a 2-deep ring, each
//           K/V tile serving both query tiles.
//   MMA issuer: ping-ponging the two query tiles: while one
//           softmax warpgroup works on its scores the tensor core runs the other
//           tile's S = Q K^T or O += P V.  P is written back into TMEM over the
//           consumed S columns (bf16 pairs) and fed to tcgen05.mma as the A operand
//           straight from TMEM, so it never touches shared memory.
//   warps 4-7 / 8-11: softmax warpgroup of query tile 0 / 1, one query row per thread
//           (TMEM lane): the thread's 128 scores come from TMEM in one round trip and
//           stay in registers for max, exp (ex2.approx, softmax scale folded into one
//           FMA), row sum and bf16 packing; O is rescaled in TMEM only when the
//           running row max grows by more than 2^8 (the stale max is exact because the
//           final normalisation uses the same reference max).
//   warp 0: TMA producer; warp 1: TMEM owner + MMA issuer; warps 2-3 idle.
#include "common/host_utils.h"
#include <cstdlib>
#include "common/ptx.cuh"
#include "common/fast_exp2.cuh"

namespace tt {
namespace attn {

constexpr int BLOCK = 128;
constexpr int THREADS = 384;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
constexpr int kDefaultVariant = 12;  // packed f32x2 softmax, 2 of every 8 exponentials on the FMA pipe

struct FwdParams {
  int B, T, Tk, Hq, Hkv;
  int q_col0, k_col0, v_col0;
  __nv_bfloat16* o;
  int ld_o;
  float* lse;
  float scale_log2;
  int causal;
  int causal_offset;  // query i attends keys j <= i + causal_offset
  int* status;
  int handoff;    // 1: the two softmax warpgroups take turns per tile (TT_ATTN_HANDOFF=1; off by default,
                  //    measured slower: 0.53 vs 0.43 ms at B4 T4096 Hq16 Hkv4 d128 causal)
  int skip_math;  // diagnostics (-DTT_ATTN_DIAGNOSTICS and TT_ATTN_SKIP_MATH=1): publish an all-zero P,
                  // to time the pipeline alone; always 0 in a production build
};

template <int D>
struct FwdSmem {
  static constexpr int TILE_BYTES = BLOCK * D * 2;
  alignas(1024) uint8_t q[2][TILE_BYTES];
  alignas(1024) uint8_t k[2][TILE_BYTES];
  alignas(1024) uint8_t v[2][TILE_BYTES];
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2], o_done[2];
  uint64_t turn[2];  // softmax hand-off: turn[x] completes when the other warpgroup finished a tile
  uint64_t done;
  uint32_t tmem_slot;
};

__device__ __forceinline__ float ex2_ftz(float x) { return ex2_mufu(x); }

// Number of 128-key tiles query tile `qt` must visit.
__device__ __forceinline__ int kv_tiles_for(const FwdParams& p, int qt) {
  if (qt * BLOCK >= p.T) return 0;
  const int n_all = (p.Tk + BLOCK - 1) / BLOCK;
  if (!p.causal) return n_all;
  const int last_q = min(qt * BLOCK + BLOCK - 1, p.T - 1) + p.causal_offset;
  return max(0, min(n_all, last_q / BLOCK + 1));
}

// VARIANT selects the softmax arithmetic mix: bit 0 = half of the exponentials on the FMA
// pipe (exp2_poly), bit 1 = bf16 packing with integer ops instead of the conversion unit,
// bit 2 = packed f32x2 math with bits 3-4 exponentials per 8 on the FMA pipe (0, 2, 3, 4).
__device__ __forceinline__ uint32_t pack_bf16x2_int(float lo, float hi) {
  // round-to-nearest (ties away from zero) of non-negative finite values, then keep the
  // high halves: (hi16(hi) << 16) | hi16(lo)
  const uint32_t a = __float_as_uint(lo) + 0x8000u;
  const uint32_t b = __float_as_uint(hi) + 0x8000u;
  return __byte_perm(a, b, 0x7632);
}

template <int D, int VARIANT>
__global__ void __launch_bounds__(THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  constexpr uint32_t TILE_BYTES = FwdSmem<D>::TILE_BYTES;
  constexpr uint32_t IDESC_QK = idesc_bf16_f32(BLOCK, BLOCK, false, false);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(BLOCK, D, false, true);
  constexpr uint32_t TMEM_COLS = 512;
  // TMEM: S/P of tile x at cols [128x, 128x+128) (P = bf16 pairs in the first 64 cols),
  //       O of tile x at cols [256 + x*D, 256 + (x+1)*D).
  auto S_COL = [](int x) { return static_cast<uint32_t>(x * BLOCK); };
  auto O_COL = [](int x) { return static_cast<uint32_t>(2 * BLOCK + x * D); };

  extern __shared__ uint8_t smem_raw[];
  FwdSmem<D>& sm = *reinterpret_cast<FwdSmem<D>*>(align_ptr(smem_raw, 1024));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_qt = (p.T + BLOCK - 1) / BLOCK;
  const int n_pairs = (n_qt + 1) / 2;
  // 1-D grid ordered tile pair slowest, (head, batch) fastest, heaviest pairs first: the block
  // scheduler hands out blocks in index order, so the long causal tiles of every head run in
  // the first wave and the short ones fill the tail (longest-first list scheduling).
  const int n_hb = p.Hq * p.B;
  const int pair = n_pairs - 1 - static_cast<int>(blockIdx.x) / n_hb;
  const int h = static_cast<int>(blockIdx.x) % p.Hq;
  const int b = (static_cast<int>(blockIdx.x) % n_hb) / p.Hq;
  const int g = h / (p.Hq / p.Hkv);
  const int k_row0 = b * p.Tk;
  int n_x[2];
  n_x[0] = kv_tiles_for(p, 2 * pair);
  n_x[1] = kv_tiles_for(p, 2 * pair + 1);
  const int n_max = max(n_x[0], n_x[1]);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.k_full[i], 1);
      mbar_init(&sm.k_empty[i], 1);
      mbar_init(&sm.v_full[i], 1);
      mbar_init(&sm.v_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], 128);
      mbar_init(&sm.o_done[i], 1);
      mbar_init(&sm.turn[i], 128);
    }
    mbar_init(&sm.done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_slot;

  if (warp == 0) {
    if (lane == 0 && n_max > 0) {
      // ------------------------------------------------ TMA producer
      mbar_arrive_expect_tx(&sm.q_full, 2 * TILE_BYTES);
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(sm.q[x] + c * BLOCK * 128, &tmQ, &sm.q_full, p.q_col0 + h * D + c * 64,
                      b * p.T + (2 * pair + x) * BLOCK);
      for (int j = 0; j < n_max; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&sm.k_empty[s], ph ^ 1u, p.status, kTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.k_full[s], TILE_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(sm.k[s] + c * BLOCK * 128, &tmK, &sm.k_full[s], p.k_col0 + g * D + c * 64, k_row0 + j * BLOCK);
        if (!mbar_wait(&sm.v_empty[s], ph ^ 1u, p.status, kTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.v_full[s], TILE_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(sm.v[s] + c * BLOCK * 128, &tmV, &sm.v_full[s], p.v_col0 + g * D + c * 64, k_row0 + j * BLOCK);
      }
      mbar_wait(&sm.q_full, 0, p.status, kTimeoutOther);
      for (int j = max(0, n_max - 2); j < n_max; ++j) {
        mbar_wait(&sm.k_full[j & 1], (j >> 1) & 1, p.status, kTimeoutOther);
        mbar_wait(&sm.v_full[j & 1], (j >> 1) & 1, p.status, kTimeoutOther);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_max > 0) {
      // ------------------------------------------------ MMA issuer (ping-pong over the two q tiles)
      auto qk = [&](int x, int j) {
        const uint32_t q_base = smem_u32(sm.q[x]);
        const uint32_t k_base = smem_u32(sm.k[j & 1]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BLOCK * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + S_COL(x), sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024),
                      IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full[x]);
      };
      auto pv = [&](int x, int j) {
        const uint32_t v_base = smem_u32(sm.v[j & 1]);
#pragma unroll
        for (int kk = 0; kk < BLOCK / 16; ++kk)  // P (A operand) read from TMEM: 8 columns per 16 keys
          umma_f16_ts(tmem + O_COL(x), tmem + S_COL(x) + kk * 8, sdesc_sw128(v_base + kk * 2048, BLOCK * 128, 1024),
                      IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&sm.o_done[x]);
      };
      bool ok = mbar_wait(&sm.q_full, 0, p.status, kTimeoutFull) &&
                mbar_wait(&sm.k_full[0], 0, p.status, kTimeoutFull);
      if (ok) {
        tc_fence_after();
        for (int x = 0; x < 2; ++x)
          if (n_x[x] > 0) qk(x, 0);
        umma_commit(&sm.k_empty[0]);
      }
      for (int j = 0; ok && j < n_max; ++j) {
        const bool next = j + 1 < n_max;
        if (!mbar_wait(&sm.v_full[j & 1], (j >> 1) & 1, p.status, kTimeoutFull)) break;
        if (next && !mbar_wait(&sm.k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, p.status, kTimeoutFull)) break;
        tc_fence_after();
        for (int x = 0; x < 2; ++x) {
          if (j < n_x[x]) {
            if (!mbar_wait(&sm.p_full[x], j & 1, p.status, kTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            pv(x, j);
          }
          if (j + 1 < n_x[x]) qk(x, j + 1);  // in-order after PV(x, j), which read P from these columns
        }
        if (!ok) break;
        umma_commit(&sm.v_empty[j & 1]);
        if (next) umma_commit(&sm.k_empty[(j + 1) & 1]);
      }
      umma_commit(&sm.done);
      mbar_wait(&sm.done, 0, p.status, kTimeoutOther);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ softmax warpgroups: x = 0 (warps 4-7), 1 (warps 8-11)
    const int x = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qt = 2 * pair + x;
    const int q_idx = qt * BLOCK + r;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + S_COL(x);
    const uint32_t o_addr = tmem + lane_addr + O_COL(x);
    const int q_lim = q_idx + p.causal_offset;
    const int n = n_x[x];
    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY;  // running max in the scaled log2 domain
    float l = 0.0f;
    bool ok = true;
    const int n_other = n_x[x ^ 1];
    for (int j = 0; j < n; ++j) {
      // With hand-off the two warpgroups alternate (A(j), B(j), A(j+1), ...) so one computes exponentials
      // while the tensor core serves the other, instead of both sharing the MUFU at once.
      const bool wait_turn = p.handoff && ((x == 0) ? (j >= 1 && j - 1 < n_other) : (j < n_other));
      const int turn_idx = (x == 0) ? j - 1 : j;
      if (wait_turn && !mbar_wait_warp(&sm.turn[x], turn_idx & 1, p.status, kTimeoutOther)) {
        ok = false;
        break;
      }
      if (!mbar_wait_warp(&sm.s_full[x], j & 1, p.status, kTimeoutAccFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
#ifdef TT_ATTN_DIAGNOSTICS
      if (p.skip_math) {  // pipeline-only timing: publish an all-zero P
#else
      if (false) {
#endif
        uint32_t z[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) z[i] = 0u;
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_st16(s_addr + c * 16, z);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.p_full[x]);
        if (p.handoff && j < n_other) mbar_arrive(&sm.turn[x ^ 1]);
        l = 1.0f;
        m_ref = 0.0f;
        continue;
      }
      const int key0 = j * BLOCK;
      const bool need_mask = (key0 + BLOCK > p.Tk) || (p.causal && key0 + BLOCK - 1 > q_lim);
      // Scores are read in 4 chunks of 32 columns, double-buffered so each chunk's TMEM
      // load overlaps the previous chunk's math.
      auto load_chunk = [&](int c, uint32_t (&buf)[32]) { tmem_ld32(s_addr + c * 32, buf); };
      auto masked = [&](uint32_t raw, int col) -> float {
        float v = __uint_as_float(raw);
        if (need_mask) {
          const int key = key0 + col;
          if (key >= p.Tk || (p.causal && key > q_lim)) v = -INFINITY;
        }
        return v;
      };
      // Exp pass with a lazily raised reference max: each 32-key chunk's max is taken first,
      // and the reference moves up only when that max exceeds it by more than 2^8, so every
      // exponential is at most 2^8 and none can overflow, however far a later key's score
      // jumps.  Chunks computed under an older reference (and the row sum and O) are rescaled
      // by 2^(m_old - m_new) afterwards; that factor may underflow to 0, which is then exact
      // in fp32.  Raising is rare after the first chunk of a row.
      const float m_start = m_ref;
      float cref[4], csum[4];
      {
        uint32_t bufA[32], bufB[32];
        load_chunk(0, bufA);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t(&cur)[32] = (c & 1) ? bufB : bufA;
          uint32_t(&nxt)[32] = (c & 1) ? bufA : bufB;
          if (c < 3) load_chunk(c + 1, nxt);
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(cur[i]);
          if (need_mask) {  // uniform per tile: only diagonal / tail tiles take this path
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int key = key0 + c * 32 + i;
              v[i] = (key >= p.Tk || (p.causal && key > q_lim)) ? -INFINITY : v[i];
            }
          }
          float e[32];
          if constexpr ((VARIANT & 4) != 0) {
            // Packed path: three-input max, f32x2 FMA for the scale, f32x2 adds for the row
            // sum, and POLY_PAIRS exponentials out of every 8 on the FMA pipe (exp2_poly2),
            // the rest on MUFU; halves the FMA/ADD issue slots so the MUFU and issue budgets
            // both stay under the tensor core's time per tile.
            constexpr int POLY = (VARIANT >> 3) & 3;  // 0: none, 1: 2 of 8, 2: 3 of 8, 3: 4 of 8
            float mq[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float m = fmax3(v[q], v[q + 4], v[q + 8]);
              m = fmax3(m, v[q + 12], v[q + 16]);
              m = fmax3(m, v[q + 20], v[q + 24]);
              mq[q] = fmaxf(m, v[q + 28]);
            }
            const float mcs = fmax3(mq[0], mq[1], fmaxf(mq[2], mq[3])) * sl2;
            if (mcs > m_ref + RESCALE_THRESHOLD) m_ref = mcs;  // also the first visible chunk (m_ref = -inf)
            const float neg_m = (m_ref == -INFINITY) ? 0.0f : -m_ref;
            const unsigned long long s2 = f2_pack(sl2, sl2), nm2 = f2_pack(neg_m, neg_m);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const unsigned long long r2 = f2_fma(f2_pack(v[i], v[i + 1]), s2, nm2);
              f2_unpack(r2, e[i], e[i + 1]);
            }
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const int w = i & 7;  // position of the pair within its group of 8
              const bool poly_pair = (POLY >= 1 && w == 6) || (POLY == 3 && w == 4);
              if (poly_pair) {
                exp2_poly2(e[i], e[i + 1]);
              } else if (POLY == 2 && w == 4) {
                e[i] = ex2_mufu(e[i]);
                e[i + 1] = exp2_poly(e[i + 1]);
              } else {
                e[i] = ex2_mufu(e[i]);
                e[i + 1] = ex2_mufu(e[i + 1]);
              }
            }
            unsigned long long sa = f2_pack(e[0], e[1]), sb = f2_pack(e[2], e[3]);
#pragma unroll
            for (int i = 4; i < 32; i += 4) {
              sa = f2_add(sa, f2_pack(e[i], e[i + 1]));
              sb = f2_add(sb, f2_pack(e[i + 2], e[i + 3]));
            }
            float a0, a1;
            f2_unpack(f2_add(sa, sb), a0, a1);
            csum[c] = a0 + a1;
          } else {
            float mq[4] = {v[0], v[1], v[2], v[3]};  // independent chains
#pragma unroll
            for (int i = 4; i < 32; i += 4) {
              mq[0] = fmaxf(mq[0], v[i]);
              mq[1] = fmaxf(mq[1], v[i + 1]);
              mq[2] = fmaxf(mq[2], v[i + 2]);
              mq[3] = fmaxf(mq[3], v[i + 3]);
            }
            const float mcs = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl2;
            if (mcs > m_ref + RESCALE_THRESHOLD) m_ref = mcs;  // also the first visible chunk (m_ref = -inf)
            const float neg_m = (m_ref == -INFINITY) ? 0.0f : -m_ref;
#pragma unroll
            for (int i = 0; i < 32; ++i) e[i] = fmaf(v[i], sl2, neg_m);
#pragma unroll
            for (int i = 0; i < 32; ++i) e[i] = ((VARIANT & 1) && (i & 1)) ? exp2_poly(e[i]) : ex2_mufu(e[i]);
            float sq[4] = {e[0], e[1], e[2], e[3]};
#pragma unroll
            for (int i = 4; i < 32; i += 4) {
              sq[0] += e[i];
              sq[1] += e[i + 1];
              sq[2] += e[i + 2];
              sq[3] += e[i + 3];
            }
            csum[c] = (sq[0] + sq[1]) + (sq[2] + sq[3]);
          }
          cref[c] = m_ref;
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = (VARIANT & 2) ? pack_bf16x2_int(e[2 * i], e[2 * i + 1]) : pack_bf16x2(e[2 * i], e[2 * i + 1]);
          tmem_st16(s_addr + c * 16, pk);
          if (c < 3) tmem_ld_wait();
        }
      }
      float rs = 0.0f;
      float cf[4];
      bool fix = false;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        cf[c] = (cref[c] == m_ref) ? 1.0f : ex2_ftz(cref[c] - m_ref);
        fix |= cf[c] != 1.0f;
        rs = fmaf(csum[c], cf[c], rs);
      }
      if (__any_sync(0xffffffffu, fix)) {  // rare, warp-collective fix-up of P chunks (factor 1 elsewhere)
        tmem_st_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pv[16];
          tmem_ld16(s_addr + c * 16, pv);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 f = unpack_bf16x2(pv[i]);
            pv[i] = pack_bf16x2(f.x * cf[c], f.y * cf[c]);
          }
          tmem_st16(s_addr + c * 16, pv);
        }
      }
      const float alpha = (m_start == m_ref) ? 1.0f : ex2_ftz(m_start - m_ref);
      l = l * alpha + rs;
      if (__any_sync(0xffffffffu, j > 0 && alpha != 1.0f)) {  // warp-collective O rescale (alpha = 1 elsewhere)
#pragma unroll
        for (int c = 0; c < D; c += 16) {
          uint32_t ov[16];
          tmem_ld16(o_addr + c, ov);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st16(o_addr + c, ov);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sm.p_full[x]);
      if (p.handoff && j < n_other) mbar_arrive(&sm.turn[x ^ 1]);
    }
    // ------------------------------------------------ epilogue: O / l, LSE
    if (ok && n > 0 && mbar_wait_warp(&sm.o_done[x], (n - 1) & 1, p.status, kTimeoutAccFull)) {
      tc_fence_after();
      const float inv_l = (l > 0.0f) ? 1.0f / l : 0.0f;
      const bool row_ok = q_idx < p.T;
      __nv_bfloat16* orow = p.o + static_cast<size_t>(b * p.T + q_idx) * p.ld_o + static_cast<size_t>(h) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t ov[32];
        tmem_ld32(o_addr + c, ov);
        tmem_ld_wait();
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(pack_bf16x2(__uint_as_float(ov[8 * i]) * inv_l, __uint_as_float(ov[8 * i + 1]) * inv_l),
                                pack_bf16x2(__uint_as_float(ov[8 * i + 2]) * inv_l, __uint_as_float(ov[8 * i + 3]) * inv_l),
                                pack_bf16x2(__uint_as_float(ov[8 * i + 4]) * inv_l, __uint_as_float(ov[8 * i + 5]) * inv_l),
                                pack_bf16x2(__uint_as_float(ov[8 * i + 6]) * inv_l, __uint_as_float(ov[8 * i + 7]) * inv_l));
        }
      }
      if (row_ok && p.lse != nullptr) {
        const float lse = (l > 0.0f) ? (m_ref + log2f(l)) * 0.69314718055994531f : -INFINITY;
        p.lse[(static_cast<size_t>(b) * p.Hq + h) * p.T + q_idx] = lse;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

CUtensorMap head_map(const torch::Tensor& t) {
  // t: [rows, cols] bf16 token-major; box {64 cols, 128 rows}
  TT_CHECK(t.dim() == 2 && t.stride(1) == 1, "attention operand must be 2-D row-major");
  return make_tmap_2d_bf16(t.data_ptr(), static_cast<uint64_t>(t.size(1)), static_cast<uint64_t>(t.size(0)),
                           static_cast<uint64_t>(t.stride(0)) * 2, 64, BLOCK);
}

}  // namespace attn

CUtensorMap attn_head_map(const torch::Tensor& t) { return attn::head_map(t); }

// q: [B*T, *] with q head h at columns q_col0 + h*D; k/v: [B*Tk, *] likewise.
// o: [B*T, >= Hq*D] bf16; lse: [B, Hq, T] fp32 (optional).
void attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t q_col0, int64_t k_col0, int64_t v_col0,
              int64_t B, int64_t T, int64_t Tk, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor o,
              c10::optional<torch::Tensor> lse, double scale, bool causal, int64_t causal_offset) {
  using namespace attn;
  check_cuda_bf16(q, "q");
  check_cuda_bf16(k, "k");
  check_cuda_bf16(v, "v");
  check_cuda_bf16(o, "o");
  TT_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TT_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TT_CHECK(q.size(0) >= B * T && k.size(0) >= B * Tk && v.size(0) >= B * Tk, "row counts");
  TT_CHECK(q_col0 % 64 == 0 && k_col0 % 64 == 0 && v_col0 % 64 == 0, "head column offsets must be 64-aligned");
  TT_CHECK(o.stride(1) == 1 && o.stride(0) % 8 == 0 && o.size(0) >= B * T && o.size(1) >= Hq * D, "o shape");
  if (lse.has_value())
    TT_CHECK(lse->scalar_type() == torch::kFloat32 && lse->numel() >= B * Hq * T, "lse must be fp32 [B,Hq,T]");
  if (B == 0 || T == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  FwdParams p{};
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.Tk = static_cast<int>(Tk);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.q_col0 = static_cast<int>(q_col0);
  p.k_col0 = static_cast<int>(k_col0);
  p.v_col0 = static_cast<int>(v_col0);
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.ld_o = static_cast<int>(o.stride(0));
  p.lse = lse.has_value() ? lse->data_ptr<float>() : nullptr;
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  p.causal_offset = static_cast<int>(causal_offset);
  p.status = device_status_ptr(q.get_device());
  {
    static const int handoff = [] { const char* e = std::getenv("TT_ATTN_HANDOFF"); return e ? std::atoi(e) : 0; }();
    p.handoff = handoff;
#ifdef TT_ATTN_DIAGNOSTICS
    static const int skip = [] { const char* e = std::getenv("TT_ATTN_SKIP_MATH"); return e ? std::atoi(e) : 0; }();
    p.skip_math = skip;
#else
    p.skip_math = 0;
#endif
  }
  const CUtensorMap tq = head_map(q), tk = head_map(k), tv = head_map(v);
  const dim3 grid(static_cast<unsigned>(((T + BLOCK - 1) / BLOCK + 1) / 2 * Hq * B));
  static const int variant = [] { const char* e = std::getenv("TT_ATTN_VARIANT"); return e ? std::atoi(e) : kDefaultVariant; }();
  auto launch = [&](auto kern, size_t smem) {
    TT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, THREADS, smem, cur_stream()>>>(tq, tk, tv, p);
  };
  if (D == 128) {
    const size_t smem = sizeof(FwdSmem<128>) + 1024;
    switch (variant) {
      case 1: launch(attn_fwd_kernel<128, 1>, smem); break;
      case 4: launch(attn_fwd_kernel<128, 4>, smem); break;
      case 12: launch(attn_fwd_kernel<128, 12>, smem); break;
      case 20: launch(attn_fwd_kernel<128, 20>, smem); break;
      case 28: launch(attn_fwd_kernel<128, 28>, smem); break;
      case 0: launch(attn_fwd_kernel<128, 0>, smem); break;
      default: launch(attn_fwd_kernel<128, kDefaultVariant>, smem); break;
    }
  } else {
    launch(attn_fwd_kernel<64, 0>, sizeof(FwdSmem<64>) + 1024);
  }
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
