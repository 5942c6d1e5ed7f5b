// Flash-attention backward on sm_100a tensor cores (tcgen05 + TMEM), GQA-native.
// Pipelined: Q/dO tiles double-buffered, P^T kept in TMEM as the A operand of the dV
// MMA, the next S^T issued while the compute warps form dS (see the kernel comment).
//
// Replaces the autograd backward of SDPA + repeat_interleave used by the reference
// (tinytron/model/modules/attn.py:66-83, 420).  One CTA owns a 128-key tile of one
// kv head and loops over every q head of its GQA group and every q tile that can
// see the keys (causal), so dK/dV for the group accumulate in TMEM and are written
// once, unexpanded.  Per (q head, q tile) iteration, five tcgen05 MMAs:
//   S^T  = K Q^T        (TMEM, lanes = keys)
//   dP^T = V dO^T       (TMEM, lanes = keys)
//   dV  += P^T dO       (P^T written back into TMEM over S^T, read as the A operand)
//   dK  += dS^T Q       (dS^T written to smem)
//   dQp  = dS K         (TMEM, lanes = queries; same smem dS^T buffer read MN-major)
// dQp is added into an fp32 accumulator with vector atomics; a final kernel
// converts it to bf16.  Inputs/outputs are token-major (packed qkv layout).
#include "common/host_utils.h"
#include <cstdlib>
#include "common/ptx.cuh"
#include "common/fast_exp2.cuh"

namespace tt {
namespace attn {

constexpr int BLOCK_B = 128;
constexpr int BWD_THREADS = 512;  // warp 0 TMA, warp 1 MMA, warps 4..11 two compute warpgroups,
                                   // warps 12..15 the dQ read-out warpgroup (warps 2-3 idle)
// Registers per thread after setmaxnreg (launch: 65536 / 512 = 128 each):
// 96 (warpgroup 0: TMA + MMA issue) + 2 x 144 (compute) + 128 (dQ) = 512 = 4 x 128.
constexpr int REG_WG0 = 96, REG_COMPUTE = 144, REG_DQ = 128;
static_assert(REG_WG0 + 2 * REG_COMPUTE + REG_DQ <= 4 * (65536 / BWD_THREADS), "register split exceeds the launch");

struct BwdParams {
  int B, T, Hq, Hkv;
  int q_col0, k_col0, v_col0, do_col0;
  const float* lse2_pad;   // [B*Hq, T_pad]  lse * log2(e), +inf past T
  const float* delta_pad;  // [B*Hq, T_pad]  rowsum(dO * O), 0 past T
  int T_pad;
  float* dq_acc;           // [B*T, Hq*D] fp32
  __nv_bfloat16* dk;       // token-major, kv head g at dk_col0 + g*D
  __nv_bfloat16* dv;
  int ld_dk, ld_dv, dk_col0, dv_col0;
  float scale;             // softmax scale
  float scale_log2;
  int causal;
  int* status;
  int dq_tma;  // 1: dQ partials reduced into dq_acc by TMA (T a multiple of 128), 0: red.v4 per thread
  int diag;  // diagnostics only, compiled in with -DTT_ATTN_DIAGNOSTICS (TT_ATTN_BWD_DIAG, wrong
             // results): 1 skips the dQ reductions, 2 skips the exponentials (P = scores), 4 skips the
             // dQ TMEM read-out entirely.  Without the macro every test below folds to false.
};

// Diagnostic bit test: constant false unless the build defines TT_ATTN_DIAGNOSTICS, so the
// production kernel carries no branch that could produce wrong gradients.
#ifdef TT_ATTN_DIAGNOSTICS
#define TT_BWD_DIAG(p, bit) (((p).diag & (bit)) != 0)
#else
#define TT_BWD_DIAG(p, bit) false
#endif

template <int D>
struct BwdSmem {
  static constexpr int TILE = BLOCK_B * D * 2;
  alignas(1024) uint8_t k[TILE];
  alignas(1024) uint8_t v[TILE];
  alignas(1024) uint8_t q[2][TILE];
  alignas(1024) uint8_t dout[2][TILE];
  alignas(1024) uint8_t dst[BLOCK_B * BLOCK_B * 2];  // dS^T [keys][queries], 128B-swizzled
  float lse2[2][BLOCK_B];                             // staged with Q/dO by the producer
  float delta[2][BLOCK_B];
  uint64_t kv_full, qdo_full[2], qdo_empty[2], s_full, p_ready, dp_full, ds_ready, dq_full, dq_empty, done;
  uint64_t stage_free;  // the dQ warpgroup finished staging through the dS^T buffer
  uint32_t tmem_slot;
};
// Bytes the layout actually uses (sizeof rounds up to the 1 KB member alignment).
template <int D>
constexpr uint32_t bwd_smem_bytes() {
  return static_cast<uint32_t>(offsetof(BwdSmem<D>, tmem_slot) + sizeof(uint32_t));
}

__device__ __forceinline__ uint32_t sw128(int row, int col, int rows) {
  const int chunk = col >> 6;
  const int unit = (col & 63) >> 3;
  return static_cast<uint32_t>(chunk * rows * 128 + row * 128 + ((unit ^ (row & 7)) << 4) + ((col & 7) << 1));
}

// One CTA per (key tile, kv head, batch); it = (q head in the group, q tile).
// MMA order (one thread):  S^T(0), dP^T(0); per it:
//   [p_ready(it)] dV += P^T(it) dO ; [next] S^T(it+1) ;
//   [ds_ready(it)] dK += dS^T Q ; dQ = dS K (into the dP^T columns) ; [dq_empty(it), next] dP^T(it+1)
// Compute warpgroups (each owns half of the query columns, then half of the head dim):
//   P(0); per it: [stage_free(it-1)] dS(it) -> ds_ready ; P(it+1) -> p_ready
// dQ warpgroup (all head dims of its 32 query rows per warp):
//   per it: [dq_full(it)] dQ read out of TMEM -> dq_empty ; staged transpose + fp32 vector
//   reductions into dq_acc -> stage_free
// so the exponentials of the next tile and the dQ read-out run side by side while the
// tensor core computes dK, dQ and the next dP^T.
template <int D>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const BwdParams p) {
  constexpr uint32_t TILE = BwdSmem<D>::TILE;
  constexpr uint32_t ID_SQ = idesc_bf16_f32(BLOCK_B, BLOCK_B, false, false);  // S^T, dP^T
  constexpr uint32_t ID_KV = idesc_bf16_f32(BLOCK_B, D, false, true);         // dV (A from TMEM), dK
  constexpr uint32_t ID_DQ = idesc_bf16_f32(BLOCK_B, D, true, true);          // dQ
  constexpr uint32_t S_COL = 0, DP_COL = BLOCK_B, DV_COL = 2 * BLOCK_B, DK_COL = 2 * BLOCK_B + D;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr int QH = BLOCK_B / 2;  // query columns per compute warpgroup
  constexpr int DH = D / 2;        // head-dim columns per compute warpgroup
  static_assert(DK_COL + D <= TMEM_COLS, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  BwdSmem<D>& sm = *reinterpret_cast<BwdSmem<D>*>(align_ptr(smem_raw, 1024));
  // The D=128 layout needs all but ~0.9 KB of the 227 KB limit, so the launch does not
  // reserve a full 1 KB for aligning the base; check that the aligned layout fits.
  if (static_cast<uint32_t>(reinterpret_cast<uint8_t*>(&sm) - smem_raw) + bwd_smem_bytes<D>() > dynamic_smem_size()) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, static_cast<int>(kSmemTooSmall));
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.T + BLOCK_B - 1) / BLOCK_B;
  // 1-D grid ordered key tile slowest, (kv head, batch) fastest: the block scheduler hands
  // out blocks in index order, so every low-kt (longest, causal) tile of every head starts in
  // the first wave and the short tiles fill the tail (longest-first list scheduling).
  const int n_gb = p.Hkv * p.B;
  const int kt = static_cast<int>(blockIdx.x) / n_gb;
  const int g = static_cast<int>(blockIdx.x) % p.Hkv;
  const int b = (static_cast<int>(blockIdx.x) % n_gb) / p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int qt0 = p.causal ? kt : 0;
  const int per_head = n_qt - qt0;
  const int n_iter = group * per_head;
  const int row0 = b * p.T;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    mbar_init(&sm.kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.qdo_full[i], 1);
      mbar_init(&sm.qdo_empty[i], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.p_ready, 256);
    mbar_init(&sm.dp_full, 1);
    mbar_init(&sm.ds_ready, 256);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_empty, 128);
    mbar_init(&sm.stage_free, 128);
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
  // Register reallocation inside each role's branch, so the compiler allocates each role
  // for its own limit (every warp of a warpgroup executes its warpgroup's instruction).
  if (warp < 4) {
  setmaxnreg_dec<REG_WG0>();
  if (warp == 0) {
    if (lane == 0 && n_iter > 0) {
      // ------------------------------------------------ producer (Q/dO/LSE/Delta double-buffered)
      mbar_arrive_expect_tx(&sm.kv_full, 2 * TILE);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sm.k + c * BLOCK_B * 128, &tmK, &sm.kv_full, p.k_col0 + g * D + c * 64, row0 + kt * BLOCK_B);
        tma_load_2d(sm.v + c * BLOCK_B * 128, &tmV, &sm.kv_full, p.v_col0 + g * D + c * 64, row0 + kt * BLOCK_B);
      }
      for (int it = 0; it < n_iter; ++it) {
        const int s = it & 1;
        const int h = g * group + it / per_head;
        const int qt = qt0 + it % per_head;
        if (!mbar_wait(&sm.qdo_empty[s], ((it >> 1) & 1) ^ 1u, p.status, kTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.qdo_full[s], 2 * TILE + 2 * BLOCK_B * 4);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(sm.q[s] + c * BLOCK_B * 128, &tmQ, &sm.qdo_full[s], p.q_col0 + h * D + c * 64,
                      row0 + qt * BLOCK_B);
          tma_load_2d(sm.dout[s] + c * BLOCK_B * 128, &tmDO, &sm.qdo_full[s], p.do_col0 + h * D + c * 64,
                      row0 + qt * BLOCK_B);
        }
        const size_t vo = (static_cast<size_t>(b) * p.Hq + h) * p.T_pad + static_cast<size_t>(qt) * BLOCK_B;
        bulk_load_1d(sm.lse2[s], p.lse2_pad + vo, BLOCK_B * 4, &sm.qdo_full[s]);
        bulk_load_1d(sm.delta[s], p.delta_pad + vo, BLOCK_B * 4, &sm.qdo_full[s]);
      }
      mbar_wait(&sm.kv_full, 0, p.status, kTimeoutOther);
      for (int it = max(0, n_iter - 2); it < n_iter; ++it)
        mbar_wait(&sm.qdo_full[it & 1], (it >> 1) & 1, p.status, kTimeoutOther);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_iter > 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t k_b = smem_u32(sm.k), v_b = smem_u32(sm.v), ds_b = smem_u32(sm.dst);
      auto s_mma = [&](int it) {  // S^T = K Q^T
        const uint32_t q_b = smem_u32(sm.q[it & 1]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BLOCK_B * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + S_COL, sdesc_sw128(k_b + off, 16, 1024), sdesc_sw128(q_b + off, 16, 1024), ID_SQ,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full);
      };
      auto dp_mma = [&](int it) {  // dP^T = V dO^T
        const uint32_t do_b = smem_u32(sm.dout[it & 1]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BLOCK_B * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + DP_COL, sdesc_sw128(v_b + off, 16, 1024), sdesc_sw128(do_b + off, 16, 1024), ID_SQ,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.dp_full);
      };
      bool ok = mbar_wait(&sm.kv_full, 0, p.status, kTimeoutFull) &&
                mbar_wait(&sm.qdo_full[0], 0, p.status, kTimeoutFull);
      if (ok) {
        tc_fence_after();
        s_mma(0);
        dp_mma(0);
      }
      for (int it = 0; ok && it < n_iter; ++it) {
        const uint32_t ph = it & 1;
        const bool next = it + 1 < n_iter;
        const uint32_t q_b = smem_u32(sm.q[it & 1]), do_b = smem_u32(sm.dout[it & 1]);
        // dV += P^T dO   (P^T in TMEM over the S^T columns, 8 columns per 16 queries)
        if (!mbar_wait(&sm.p_ready, ph, p.status, kTimeoutFull)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BLOCK_B / 16; ++kk)
          umma_f16_ts(tmem + DV_COL, tmem + S_COL + kk * 8, sdesc_sw128(do_b + kk * 2048, BLOCK_B * 128, 1024),
                      ID_KV, (it > 0 || kk > 0) ? 1u : 0u);
        if (next) {  // next scores, in order after the dV MMA that reads P^T from the same columns
          if (!mbar_wait(&sm.qdo_full[(it + 1) & 1], ((it + 1) >> 1) & 1, p.status, kTimeoutFull)) break;
          tc_fence_after();
          s_mma(it + 1);
        }
        // dK += dS^T Q ; dQ = dS K (into the consumed dP^T columns)
        if (!mbar_wait(&sm.ds_ready, ph, p.status, kTimeoutFull)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BLOCK_B / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * (BLOCK_B * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + DK_COL, sdesc_sw128(ds_b + a_off, 16, 1024),
                      sdesc_sw128(q_b + kk * 2048, BLOCK_B * 128, 1024), ID_KV, (it > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < BLOCK_B / 16; ++kk)
          umma_f16_ss(tmem + DP_COL, sdesc_sw128(ds_b + kk * 2048, BLOCK_B * 128, 1024),
                      sdesc_sw128(k_b + kk * 2048, BLOCK_B * 128, 1024), ID_DQ, kk > 0 ? 1u : 0u);
        umma_commit(&sm.dq_full);  // also tells the compute warps that dS^T in smem is consumed
        umma_commit(&sm.qdo_empty[it & 1]);
        if (next) {
          if (!mbar_wait(&sm.dq_empty, ph, p.status, kTimeoutAccEmpty)) break;
          tc_fence_after();
          dp_mma(it + 1);
        }
      }
      umma_commit(&sm.done);
      mbar_wait(&sm.done, 0, p.status, kTimeoutOther);
    }
  }  // warps 2-3: idle
  } else if (warp < 12) {
    setmaxnreg_inc<REG_COMPUTE>();
    // ------------------------------------------------ compute warps 4..11
    const int half = (warp - 4) >> 2;   // warpgroup: query columns [half*64, +64), head dims [half*D/2, +D/2)
    const int quarter = warp & 3;       // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;  // key row (P / dS phases), query row (dQ phase)
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int key = kt * BLOCK_B + r;
    const float key_scale = (key < p.T) ? 1.0f : 0.0f;  // keys past the end were masked in forward
    float pv[QH];
    // P^T row (this warpgroup's 64 queries) = 2^(S^T * scale_log2 - lse2[q]); causal diagonal:
    // queries before the key are 0.  Written back into TMEM as bf16 pairs over S^T.
    auto p_phase = [&](int it) -> bool {
      const int qt = qt0 + it % per_head;
      const int buf = it & 1;
      if (!mbar_wait_warp(&sm.s_full, it & 1, p.status, kTimeoutAccFull)) return false;
      if (!mbar_wait_warp(&sm.qdo_full[buf], (it >> 1) & 1, p.status, kTimeoutFull)) return false;  // lse2 landed
      tc_fence_after();
      uint32_t raw[QH];
      tmem_ld32(tmem + lane_addr + S_COL + half * QH, *reinterpret_cast<uint32_t(*)[32]>(&raw[0]));
      tmem_ld32(tmem + lane_addr + S_COL + half * QH + 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[32]));
      tmem_ld_wait();
      const float* l2 = sm.lse2[buf] + half * QH;
#pragma unroll
      for (int i = 0; i < QH; ++i) pv[i] = ex2_mufu(fmaf(__uint_as_float(raw[i]), p.scale_log2, -l2[i])) * key_scale;
      if (TT_BWD_DIAG(p, 2)) {
#pragma unroll
        for (int i = 0; i < QH; ++i) pv[i] = __uint_as_float(raw[i]) * key_scale;
      }
      if (p.causal && qt == kt) {
#pragma unroll
        for (int i = 0; i < QH; ++i) pv[i] = (half * QH + i < r) ? 0.0f : pv[i];
      }
#pragma unroll
      for (int c = 0; c < QH; c += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(pv[c + 2 * i], pv[c + 2 * i + 1]);
        tmem_st16(tmem + lane_addr + S_COL + ((half * QH + c) >> 1), pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sm.p_ready);
      return true;
    };
    bool ok = n_iter > 0 && p_phase(0);
    for (int it = 0; ok && it < n_iter; ++it) {
      const uint32_t ph = it & 1;
      const int buf = it & 1;
      // ---- dS^T = P^T * (dP^T - delta[q]) * scale -> shared memory (A of dK, MN-major A of dQ).
      // dp_full(it) follows dK/dQ(it-1), the MMAs that read the previous dS^T.
      if (!mbar_wait_warp(&sm.dp_full, ph, p.status, kTimeoutAccFull)) { ok = false; break; }
      // the dQ warpgroup's staging of the previous iteration must be out of the dS^T buffer
      if (it > 0 && !mbar_wait_warp(&sm.stage_free, (it - 1) & 1, p.status, kTimeoutOther)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t d0[32], d1[32];
        tmem_ld32(tmem + lane_addr + DP_COL + half * QH, d0);
        tmem_ld32(tmem + lane_addr + DP_COL + half * QH + 32, d1);
        tmem_ld_wait();
        const float* dl = sm.delta[buf] + half * QH;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint32_t(&cur)[32] = c ? d1 : d0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float ds[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int j = c * 32 + 8 * u + i;
              ds[i] = pv[j] * (__uint_as_float(cur[8 * u + i]) - dl[j]) * p.scale;
            }
            const uint4 w = make_uint4(pack_bf16x2(ds[0], ds[1]), pack_bf16x2(ds[2], ds[3]),
                                       pack_bf16x2(ds[4], ds[5]), pack_bf16x2(ds[6], ds[7]));
            *reinterpret_cast<uint4*>(sm.dst + sw128(r, half * QH + c * 32 + 8 * u, BLOCK_B)) = w;
          }
        }
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.ds_ready);
      // ---- next tile's probabilities while dK / dQ run on the tensor core
      if (it + 1 < n_iter && !p_phase(it + 1)) { ok = false; break; }
    }
    // ---- dK, dV (lane = key row), this warpgroup's head-dim half -> bf16
    if (ok && n_iter > 0 && mbar_wait_warp(&sm.done, 0, p.status, kTimeoutAccFull)) {
      tc_fence_after();
      const bool key_ok = key < p.T;
      __nv_bfloat16* dkrow =
          p.dk + static_cast<size_t>(row0 + key) * p.ld_dk + p.dk_col0 + static_cast<size_t>(g) * D + half * DH;
      __nv_bfloat16* dvrow =
          p.dv + static_cast<size_t>(row0 + key) * p.ld_dv + p.dv_col0 + static_cast<size_t>(g) * D + half * DH;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = (which == 0 ? DK_COL : DV_COL) + half * DH;
        __nv_bfloat16* out = which == 0 ? dkrow : dvrow;
#pragma unroll
        for (int c = 0; c < DH; c += 32) {
          uint32_t rr[32];
          tmem_ld32(tmem + lane_addr + col + c, rr);
          tmem_ld_wait();
          if (key_ok) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<uint4*>(out + c)[i] =
                  make_uint4(pack_bf16x2(__uint_as_float(rr[8 * i]), __uint_as_float(rr[8 * i + 1])),
                             pack_bf16x2(__uint_as_float(rr[8 * i + 2]), __uint_as_float(rr[8 * i + 3])),
                             pack_bf16x2(__uint_as_float(rr[8 * i + 4]), __uint_as_float(rr[8 * i + 5])),
                             pack_bf16x2(__uint_as_float(rr[8 * i + 6]), __uint_as_float(rr[8 * i + 7])));
          }
        }
      }
    }
  } else {
    setmaxnreg_dec<REG_DQ>();
    // ------------------------------------------------ dQ warpgroup (warps 12..15)
    // Per iteration: dQ(it) (128 queries x D, in the dP^T columns) is read out of TMEM,
    // the columns released (dq_empty) as soon as every value is in registers, then each
    // 32x32 block is transposed through this warp's 4 KB slice of the dS^T buffer so every
    // red.v4 instruction covers four whole 128-byte rows of dq_acc instead of 32 scattered
    // 16-byte pieces; stage_free then lets the compute warps write the next dS^T.
    const int quarter = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    // Staging: two 4 KB slices of the dS^T buffer per warp (1 KB aligned, laid out with the
    // 128-byte swizzle the TMA reduction reads), alternating per 32-column block.
    uint8_t* stage0 = sm.dst + quarter * 2 * 4096;
    for (int it = 0; it < n_iter; ++it) {
      const int h = g * group + it / per_head;
      const int qt = qt0 + it % per_head;
      if (!mbar_wait_warp(&sm.dq_full, it & 1, p.status, kTimeoutAccFull)) break;
      tc_fence_after();
      if (TT_BWD_DIAG(p, 4)) {  // diagnostics: skip the read-out
        tc_fence_before();
        mbar_arrive(&sm.dq_empty);
        mbar_arrive(&sm.stage_free);
        continue;
      }
      const int qbase = qt * BLOCK_B + quarter * 32;  // query of this warp's first row
      float* gbase = p.dq_acc + static_cast<size_t>(row0) * (p.Hq * D) + static_cast<size_t>(h) * D;
#pragma unroll
      for (int c2 = 0; c2 < D / 64; ++c2) {
        uint32_t cur[2][32];
        tmem_ld32(tmem + lane_addr + DP_COL + c2 * 64, cur[0]);
        tmem_ld32(tmem + lane_addr + DP_COL + c2 * 64 + 32, cur[1]);
        tmem_ld_wait();
        if (c2 == D / 64 - 1) {
          tc_fence_before();
          mbar_arrive(&sm.dq_empty);  // all values are in registers: the dP^T columns are free again
        }
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          const int blk = c2 * 2 + hb;  // 32-column block of the head dim
          uint8_t* stage = stage0 + (blk & 1) * 4096;
          if (p.dq_tma && blk >= 2) {  // the reduction issued two blocks ago has read this slice
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
          }
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((u ^ (lane & 7)) << 4)) =
                make_uint4(cur[hb][4 * u], cur[hb][4 * u + 1], cur[hb][4 * u + 2], cur[hb][4 * u + 3]);
          if (p.dq_tma) {
            fence_proxy_async();
            __syncwarp();
            if (lane == 0 && !TT_BWD_DIAG(p, 1)) {
              tma_reduce_add_2d(&tmDQ, stage, h * D + blk * 32, row0 + qbase);
              bulk_commit_group();
            }
          } else {
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int j = i * 4 + (lane >> 3);  // row within the warp's 32
              const int u = lane & 7;             // 16-byte unit within the 32 columns
              const float4 v = *reinterpret_cast<const float4*>(stage + j * 128 + ((u ^ (j & 7)) << 4));
              if (qbase + j < p.T && !TT_BWD_DIAG(p, 1))
                atomicAdd(reinterpret_cast<float4*>(gbase + static_cast<size_t>(qbase + j) * (p.Hq * D) + blk * 32) + u,
                          v);
            }
            __syncwarp();
          }
        }
      }
      if (p.dq_tma) {  // the staging slices are read before the compute warps may overwrite them
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
      }
      mbar_arrive(&sm.stage_free);
    }
    if (p.dq_tma) {  // every reduction performed before the block exits
      if (lane == 0) bulk_wait_group<0>();
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// Per (b, h, t < T_pad): delta = sum_d dO[t, h*D + d] * O[t, h*D + d] and lse2 = lse * log2(e);
// padded positions t >= T get delta 0 and lse2 +inf (their probabilities become 0).
// One warp per (token slot, head).
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, int ld_o, const __nv_bfloat16* __restrict__ dout,
                                      int ld_do, const float* __restrict__ lse, float* __restrict__ lse2_pad,
                                      float* __restrict__ delta_pad, int B, int T, int T_pad, int Hq, int D) {
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(B) * T_pad * Hq;
  if (wid >= total) return;
  const int h = static_cast<int>(wid % Hq);
  const long long slot = wid / Hq;
  const int b = static_cast<int>(slot / T_pad), t = static_cast<int>(slot % T_pad);
  const size_t out = (static_cast<size_t>(b) * Hq + h) * T_pad + t;
  if (t >= T) {
    if (lane == 0) {
      delta_pad[out] = 0.0f;
      lse2_pad[out] = INFINITY;
    }
    return;
  }
  const long long tok = static_cast<long long>(b) * T + t;
  const __nv_bfloat16* a = o + tok * ld_o + static_cast<long long>(h) * D;
  const __nv_bfloat16* c = dout + tok * ld_do + static_cast<long long>(h) * D;
  float s = 0.0f;
  for (int i = lane * 4; i < D; i += 128) {
    const uint2 x = *reinterpret_cast<const uint2*>(a + i);
    const uint2 y = *reinterpret_cast<const uint2*>(c + i);
    const float2 x0 = unpack_bf16x2(x.x), x1 = unpack_bf16x2(x.y), y0 = unpack_bf16x2(y.x), y1 = unpack_bf16x2(y.y);
    s += x0.x * y0.x + x0.y * y0.y + x1.x * y1.x + x1.y * y1.y;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    delta_pad[out] = s;
    lse2_pad[out] = lse[(static_cast<size_t>(b) * Hq + h) * T + t] * 1.4426950408889634f;
  }
}

// Same outputs, one warp per token covering all heads (Hq * D a multiple of 256, D = 64 or
// 128): lane l reads 16-byte chunks l + 32 j of O and dO, the D/8 lanes of a head reduce by
// shuffles.  32-bit index math; each warp streams 2 x Hq x D x 2 bytes.
__global__ void attn_bwd_delta_rows_kernel(const __nv_bfloat16* __restrict__ o, int ld_o,
                                           const __nv_bfloat16* __restrict__ dout, int ld_do,
                                           const float* __restrict__ lse, float* __restrict__ lse2_pad,
                                           float* __restrict__ delta_pad, int B, int T, int T_pad, int Hq, int D) {
  const int warp = static_cast<int>((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= B * T_pad) return;
  const int b = warp / T_pad, t = warp - (warp / T_pad) * T_pad;
  if (t >= T) {  // padded slots
    for (int h = lane; h < Hq; h += 32) {
      const int out = (b * Hq + h) * T_pad + t;
      delta_pad[out] = 0.0f;
      lse2_pad[out] = INFINITY;
    }
    return;
  }
  const int tok = b * T + t;
  const uint4* a = reinterpret_cast<const uint4*>(o + static_cast<long long>(tok) * ld_o);
  const uint4* c = reinterpret_cast<const uint4*>(dout + static_cast<long long>(tok) * ld_do);
  const int lanes_per_head = D / 8;  // 16 or 8
  const int n_iter = Hq * D / 256;
  for (int j = 0; j < n_iter; ++j) {
    const int chunk = lane + 32 * j;
    const uint4 x = a[chunk];
    const uint4 y = c[chunk];
    const uint32_t* xv = reinterpret_cast<const uint32_t*>(&x);
    const uint32_t* yv = reinterpret_cast<const uint32_t*>(&y);
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 xf = unpack_bf16x2(xv[q]), yf = unpack_bf16x2(yv[q]);
      s += xf.x * yf.x + xf.y * yf.y;
    }
    for (int off = lanes_per_head / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((lane & (lanes_per_head - 1)) == 0) {
      const int h = chunk / lanes_per_head;
      const int out = (b * Hq + h) * T_pad + t;
      delta_pad[out] = s;
      lse2_pad[out] = lse[(b * Hq + h) * T + t] * 1.4426950408889634f;
    }
  }
}

// dq (bf16, token-major, head h at col0 + h*D) = dq_acc (fp32 [tokens, Hq*D])
__global__ void attn_bwd_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int ld_dq,
                                           int col0, long long tokens, int width) {
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= tokens * width) return;
  const long long tok = i / width;
  const int c = static_cast<int>(i % width);
  const float4 a = reinterpret_cast<const float4*>(acc + i)[0];
  const float4 b = reinterpret_cast<const float4*>(acc + i)[1];
  *reinterpret_cast<uint4*>(dq + tok * ld_dq + col0 + c) =
      make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
}

}  // namespace attn

CUtensorMap attn_head_map(const torch::Tensor& t);

// Backward of attn_fwd (causal or full, self-attention T == Tk).
//   q/k/v/o/dout: token-major bf16 buffers with head column offsets; lse [B,Hq,T] (from fwd).
//   dq/dk/dv: token-major bf16 outputs (may all be the same packed dqkv buffer).
//   dq_acc: fp32 scratch [B*T, Hq*D]; scratch: fp32, attn_bwd_scratch_numel(B, Hq, T) elements.
void attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
              int64_t q_col0, int64_t k_col0, int64_t v_col0, torch::Tensor lse, int64_t B, int64_t T, int64_t Hq,
              int64_t Hkv, int64_t D, torch::Tensor dq, int64_t dq_col0, torch::Tensor dk, int64_t dk_col0,
              torch::Tensor dv, int64_t dv_col0, torch::Tensor dq_acc, torch::Tensor scratch, double scale,
              bool causal) {
  using namespace attn;
  for (auto* tp : {&q, &k, &v, &o, &dout, &dq, &dk, &dv}) check_cuda_bf16(*tp, "attn_bwd operand");
  TT_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TT_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TT_CHECK(dq_acc.scalar_type() == torch::kFloat32 && dq_acc.is_contiguous() && dq_acc.numel() >= B * T * Hq * D,
           "dq_acc must be fp32 [B*T, Hq*D]");
  const int64_t T_pad = (T + BLOCK_B - 1) / BLOCK_B * BLOCK_B;
  TT_CHECK(scratch.scalar_type() == torch::kFloat32 && scratch.is_contiguous() && scratch.numel() >= 2 * B * Hq * T_pad &&
               reinterpret_cast<uintptr_t>(scratch.data_ptr()) % 16 == 0,
           "scratch must be fp32 with attn_bwd_scratch_numel(B, Hq, T) elements");
  TT_CHECK(lse.scalar_type() == torch::kFloat32 && lse.numel() >= B * Hq * T, "lse must be fp32");
  TT_CHECK(q_col0 % 64 == 0 && k_col0 % 64 == 0 && v_col0 % 64 == 0, "column offsets must be 64-aligned");
  TT_CHECK(o.stride(1) == 1 && dout.stride(1) == 1 && dout.is_contiguous() == dout.is_contiguous(), "layouts");
  TT_CHECK(dq_col0 % 8 == 0 && dk_col0 % 8 == 0 && dv_col0 % 8 == 0 && dq.stride(0) % 8 == 0 &&
               dk.stride(0) % 8 == 0 && dv.stride(0) % 8 == 0,
           "output alignment");
  if (B == 0 || T == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = cur_stream();
  const long long tokens = B * T;
  float* lse2_pad = scratch.data_ptr<float>();
  float* delta_pad = lse2_pad + B * Hq * T_pad;
  const bool rows_ok = (D == 64 || D == 128) && (Hq * D) % 256 == 0 && o.stride(0) % 8 == 0 &&
                       dout.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(o.data_ptr()) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(dout.data_ptr()) % 16 == 0 && B * T_pad * Hq < (1LL << 31);
  if (rows_ok) {
    const long long warps = B * T_pad;
    attn_bwd_delta_rows_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), static_cast<int>(o.stride(0)),
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), static_cast<int>(dout.stride(0)), lse.data_ptr<float>(),
        lse2_pad, delta_pad, static_cast<int>(B), static_cast<int>(T), static_cast<int>(T_pad), static_cast<int>(Hq),
        static_cast<int>(D));
    TT_CUDA_CHECK(cudaGetLastError());
  } else {
    const long long warps = B * T_pad * Hq;
    attn_bwd_delta_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), static_cast<int>(o.stride(0)),
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), static_cast<int>(dout.stride(0)), lse.data_ptr<float>(),
        lse2_pad, delta_pad, static_cast<int>(B), static_cast<int>(T), static_cast<int>(T_pad), static_cast<int>(Hq),
        static_cast<int>(D));
    TT_CUDA_CHECK(cudaGetLastError());
  }
  TT_CUDA_CHECK(cudaMemsetAsync(dq_acc.data_ptr(), 0, static_cast<size_t>(tokens * Hq * D) * sizeof(float), st));
  BwdParams p{};
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.q_col0 = static_cast<int>(q_col0);
  p.k_col0 = static_cast<int>(k_col0);
  p.v_col0 = static_cast<int>(v_col0);
  p.do_col0 = 0;
  p.lse2_pad = lse2_pad;
  p.delta_pad = delta_pad;
  p.T_pad = static_cast<int>(T_pad);
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.ld_dk = static_cast<int>(dk.stride(0));
  p.ld_dv = static_cast<int>(dv.stride(0));
  p.dk_col0 = static_cast<int>(dk_col0);
  p.dv_col0 = static_cast<int>(dv_col0);
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  p.status = device_status_ptr(q.get_device());
#ifdef TT_ATTN_DIAGNOSTICS
  {
    static const int diag = [] { const char* e = std::getenv("TT_ATTN_BWD_DIAG"); return e ? std::atoi(e) : 0; }();
    p.diag = diag;
  }
#else
  p.diag = 0;
#endif
  const CUtensorMap tq = attn_head_map(q), tk = attn_head_map(k), tv = attn_head_map(v), tdo = attn_head_map(dout);
  // TT_ATTN_DQ_TMA=1: dQ partials are added by TMA tile reductions of 32 queries x 32 dims
  // (only when no tile can reach past the end of a sequence: T a multiple of 128).  Off by
  // default: measured slower than the per-thread red.v4 path (1.029 vs 1.005 ms backward at
  // B4 T4096 Hq16 Hkv4 d128).
  static const bool dq_tma_env = [] { const char* e = std::getenv("TT_ATTN_DQ_TMA"); return e && std::atoi(e) != 0; }();
  p.dq_tma = (dq_tma_env && T % BLOCK_B == 0) ? 1 : 0;
  const CUtensorMap tdq = make_tmap_2d_f32(dq_acc.data_ptr(), static_cast<uint64_t>(Hq * D),
                                           static_cast<uint64_t>(B * T), static_cast<uint64_t>(Hq * D * 4), 32, 32);
  const dim3 grid(static_cast<unsigned>((T + BLOCK_B - 1) / BLOCK_B * Hkv * B));
  if (D == 128) {
    const size_t smem = std::min<size_t>(bwd_smem_bytes<128>() + 1024, size_t(232448));
    TT_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_bwd_kernel<128><<<grid, BWD_THREADS, smem, st>>>(tq, tk, tv, tdo, tdq, p);
  } else {
    const size_t smem = std::min<size_t>(bwd_smem_bytes<64>() + 1024, size_t(232448));
    TT_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_bwd_kernel<64><<<grid, BWD_THREADS, smem, st>>>(tq, tk, tv, tdo, tdq, p);
  }
  TT_CUDA_CHECK(cudaGetLastError());
  const int width = static_cast<int>(Hq * D);
  const long long vecs = tokens * width / 8;
  attn_bwd_dq_convert_kernel<<<static_cast<unsigned>((vecs + 255) / 256), 256, 0, st>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), static_cast<int>(dq.stride(0)),
      static_cast<int>(dq_col0), tokens, width);
  TT_CUDA_CHECK(cudaGetLastError());
}

int64_t attn_bwd_scratch_numel(int64_t B, int64_t Hq, int64_t T) {
  return 2 * B * Hq * ((T + attn::BLOCK_B - 1) / attn::BLOCK_B * attn::BLOCK_B);
}

}  // namespace tt
