// Flash-attention backward on sm_100a tensor cores (tcgen05 + TMEM), GQA-native.
//
// Replaces the autograd backward of SDPA + repeat_interleave used by the reference
// (tinytron/model/modules/attn.py:66-83, 420).  One CTA owns a 128-key tile of one
// kv head and loops over every q head of its GQA group and every q tile that can
// see the keys (causal), so dK/dV for the group accumulate in TMEM and are written
// once, unexpanded.  Per (q head, q tile) iteration, five tcgen05 MMAs:
//   S^T  = K Q^T        (TMEM, lanes = keys)
//   dP^T = V dO^T       (TMEM, lanes = keys)
//   dV  += P^T dO       (P^T written to smem by the softmax threads)
//   dK  += dS^T Q       (dS^T written to smem)
//   dQp  = dS K         (TMEM, lanes = queries; same smem dS^T buffer read MN-major)
// dQp is added into an fp32 accumulator with vector atomics; a final kernel
// converts it to bf16.  Inputs/outputs are token-major (packed qkv layout).
#include "common/host_utils.h"
#include "common/ptx.cuh"

namespace tt {
namespace attn {

constexpr int BLOCK_B = 128;
constexpr int BWD_THREADS = 192;

struct BwdParams {
  int B, T, Hq, Hkv;
  int q_col0, k_col0, v_col0, do_col0;
  const float* lse;    // [B, Hq, T] natural log
  const float* delta;  // [B, Hq, T]  rowsum(dO * O)
  float* dq_acc;       // [B*T, Hq*D] fp32
  __nv_bfloat16* dk;   // token-major, kv head g at dk_col0 + g*D
  __nv_bfloat16* dv;
  int ld_dk, ld_dv, dk_col0, dv_col0;
  float scale;         // softmax scale
  float scale_log2;
  int causal;
  int* status;
};

template <int D>
struct BwdSmem {
  static constexpr int TILE = BLOCK_B * D * 2;
  alignas(1024) uint8_t k[TILE];
  alignas(1024) uint8_t v[TILE];
  alignas(1024) uint8_t q[TILE];
  alignas(1024) uint8_t dout[TILE];
  alignas(1024) uint8_t pt[BLOCK_B * BLOCK_B * 2];
  alignas(1024) uint8_t dst[BLOCK_B * BLOCK_B * 2];
  float lse2[2][BLOCK_B];
  float delta[2][BLOCK_B];
  uint64_t kv_full, qdo_full, qdo_empty, s_full, dp_full, dp_empty, p_ready, ds_ready, ps_free, dq_full, dq_empty,
      done, stage_bar[2];
  uint32_t tmem_slot;
};

__device__ __forceinline__ uint32_t sw128(int row, int col, int rows) {
  const int chunk = col >> 6;
  const int unit = (col & 63) >> 3;
  return static_cast<uint32_t>(chunk * rows * 128 + row * 128 + ((unit ^ (row & 7)) << 4) + ((col & 7) << 1));
}

template <int D>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const BwdParams p) {
  constexpr uint32_t TILE = BwdSmem<D>::TILE;
  constexpr uint32_t ID_SQ = idesc_bf16_f32(BLOCK_B, BLOCK_B, false, false);  // S^T, dP^T
  constexpr uint32_t ID_KV = idesc_bf16_f32(BLOCK_B, D, false, true);         // dV, dK
  constexpr uint32_t ID_DQ = idesc_bf16_f32(BLOCK_B, D, true, true);          // dQ
  constexpr uint32_t S_COL = 0, DP_COL = BLOCK_B, DV_COL = 2 * BLOCK_B, DK_COL = 2 * BLOCK_B + D;
  constexpr uint32_t TMEM_COLS = 512;
  static_assert(DK_COL + D <= TMEM_COLS, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  BwdSmem<D>& sm = *reinterpret_cast<BwdSmem<D>*>(align_ptr(smem_raw, 1024));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.T + BLOCK_B - 1) / BLOCK_B;
  const int kt = static_cast<int>(blockIdx.x);  // low kt = most work; launched first
  const int g = blockIdx.y;
  const int b = blockIdx.z;
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
    mbar_init(&sm.qdo_full, 1);
    mbar_init(&sm.qdo_empty, 1);
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.dp_full, 1);
    mbar_init(&sm.dp_empty, 128);
    mbar_init(&sm.p_ready, 128);
    mbar_init(&sm.ds_ready, 128);
    mbar_init(&sm.ps_free, 1);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_empty, 128);
    mbar_init(&sm.done, 1);
    mbar_init(&sm.stage_bar[0], 128);
    mbar_init(&sm.stage_bar[1], 128);
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
    if (lane == 0 && n_iter > 0) {
      // ------------------------------------------------ producer
      mbar_arrive_expect_tx(&sm.kv_full, 2 * TILE);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sm.k + c * BLOCK_B * 128, &tmK, &sm.kv_full, p.k_col0 + g * D + c * 64, row0 + kt * BLOCK_B);
        tma_load_2d(sm.v + c * BLOCK_B * 128, &tmV, &sm.kv_full, p.v_col0 + g * D + c * 64, row0 + kt * BLOCK_B);
      }
      for (int it = 0; it < n_iter; ++it) {
        const int h = g * group + it / per_head;
        const int qt = qt0 + it % per_head;
        if (!mbar_wait(&sm.qdo_empty, (it & 1) ^ 1u, p.status, kTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.qdo_full, 2 * TILE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_2d(sm.q + c * BLOCK_B * 128, &tmQ, &sm.qdo_full, p.q_col0 + h * D + c * 64, row0 + qt * BLOCK_B);
          tma_load_2d(sm.dout + c * BLOCK_B * 128, &tmDO, &sm.qdo_full, p.do_col0 + h * D + c * 64,
                      row0 + qt * BLOCK_B);
        }
      }
      mbar_wait(&sm.kv_full, 0, p.status, kTimeoutOther);
      mbar_wait(&sm.qdo_full, (n_iter - 1) & 1, p.status, kTimeoutOther);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_iter > 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t k_b = smem_u32(sm.k), v_b = smem_u32(sm.v), q_b = smem_u32(sm.q), do_b = smem_u32(sm.dout);
      const uint32_t pt_b = smem_u32(sm.pt), ds_b = smem_u32(sm.dst);
      bool ok = mbar_wait(&sm.kv_full, 0, p.status, kTimeoutFull);
      for (int it = 0; ok && it < n_iter; ++it) {
        const uint32_t ph = it & 1;
        if (!mbar_wait(&sm.qdo_full, ph, p.status, kTimeoutFull)) break;
        if (!mbar_wait(&sm.dq_empty, ph ^ 1u, p.status, kTimeoutAccEmpty)) break;
        tc_fence_after();
        // S^T = K Q^T
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BLOCK_B * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + S_COL, sdesc_sw128(k_b + off, 16, 1024), sdesc_sw128(q_b + off, 16, 1024), ID_SQ,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full);
        if (!mbar_wait(&sm.dp_empty, ph ^ 1u, p.status, kTimeoutAccEmpty)) break;
        tc_fence_after();
        // dP^T = V dO^T
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BLOCK_B * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + DP_COL, sdesc_sw128(v_b + off, 16, 1024), sdesc_sw128(do_b + off, 16, 1024), ID_SQ,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.dp_full);
        // dV += P^T dO
        if (!mbar_wait(&sm.p_ready, ph, p.status, kTimeoutFull)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BLOCK_B / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * (BLOCK_B * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + DV_COL, sdesc_sw128(pt_b + a_off, 16, 1024),
                      sdesc_sw128(do_b + kk * 2048, BLOCK_B * 128, 1024), ID_KV, (it > 0 || kk > 0) ? 1u : 0u);
        }
        // dK += dS^T Q ; dQp = dS K
        if (!mbar_wait(&sm.ds_ready, ph, p.status, kTimeoutFull)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BLOCK_B / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * (BLOCK_B * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + DK_COL, sdesc_sw128(ds_b + a_off, 16, 1024),
                      sdesc_sw128(q_b + kk * 2048, BLOCK_B * 128, 1024), ID_KV, (it > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < BLOCK_B / 16; ++kk) {
          umma_f16_ss(tmem + S_COL, sdesc_sw128(ds_b + kk * 2048, BLOCK_B * 128, 1024),
                      sdesc_sw128(k_b + kk * 2048, BLOCK_B * 128, 1024), ID_DQ, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.qdo_empty);
        umma_commit(&sm.ps_free);
        umma_commit(&sm.dq_full);
      }
      umma_commit(&sm.done);
      mbar_wait(&sm.done, 0, p.status, kTimeoutOther);
    }
  } else {
    // ------------------------------------------------ compute threads (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane: key row (S/dP phases), query row (dQ phase)
    const int t = threadIdx.x - 64;     // 0..127
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int key = kt * BLOCK_B + r;
    bool ok = n_iter > 0;
    for (int it = 0; ok && it < n_iter; ++it) {
      const uint32_t ph = it & 1;
      const int h = g * group + it / per_head;
      const int qt = qt0 + it % per_head;
      const int buf = it & 1;
      {  // stage this q tile's LSE (log2 domain) and Delta in shared memory
        const int q = qt * BLOCK_B + t;
        const size_t idx = (static_cast<size_t>(b) * p.Hq + h) * p.T + q;
        sm.lse2[buf][t] = (q < p.T) ? p.lse[idx] * 1.4426950408889634f : INFINITY;
        sm.delta[buf][t] = (q < p.T) ? p.delta[idx] : 0.0f;
      }
      mbar_arrive(&sm.stage_bar[buf]);
      if (!mbar_wait_warp(&sm.stage_bar[buf], (it >> 1) & 1, p.status, kTimeoutOther)) { ok = false; break; }
      // ---- P^T = exp2(S^T * scale_log2 - lse2[q]) (0 for masked / padded queries)
      if (!mbar_wait_warp(&sm.s_full, ph, p.status, kTimeoutAccFull)) { ok = false; break; }
      tc_fence_after();
      float pv[BLOCK_B];
#pragma unroll
      for (int c = 0; c < BLOCK_B; c += 32) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_addr + S_COL + c, rr);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) pv[c + i] = __uint_as_float(rr[i]);
      }
      const bool diag = p.causal && qt == kt;
      const bool key_pad = key >= p.T;  // rows past the sequence end were masked in forward
#pragma unroll
      for (int i = 0; i < BLOCK_B; ++i) {
        float e = exp2f(pv[i] * p.scale_log2 - sm.lse2[buf][i]);
        if ((diag && i < r) || key_pad) e = 0.0f;  // causal: query qt*128+i < key kt*128+r
        pv[i] = e;
      }
      if (it > 0 && !mbar_wait_warp(&sm.ps_free, ph ^ 1u, p.status, kTimeoutAccEmpty)) { ok = false; break; }
#pragma unroll
      for (int c = 0; c < BLOCK_B; c += 8) {
        const uint4 v = make_uint4(pack_bf16x2(pv[c], pv[c + 1]), pack_bf16x2(pv[c + 2], pv[c + 3]),
                                   pack_bf16x2(pv[c + 4], pv[c + 5]), pack_bf16x2(pv[c + 6], pv[c + 7]));
        *reinterpret_cast<uint4*>(sm.pt + sw128(r, c, BLOCK_B)) = v;
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.p_ready);
      // ---- dS^T = P^T * (dP^T - delta[q]) * scale
      if (!mbar_wait_warp(&sm.dp_full, ph, p.status, kTimeoutAccFull)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < BLOCK_B; c += 32) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_addr + DP_COL + c, rr);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) pv[c + i] = pv[c + i] * (__uint_as_float(rr[i]) - sm.delta[buf][c + i]) * p.scale;
      }
      tc_fence_before();
      mbar_arrive(&sm.dp_empty);
#pragma unroll
      for (int c = 0; c < BLOCK_B; c += 8) {
        const uint4 v = make_uint4(pack_bf16x2(pv[c], pv[c + 1]), pack_bf16x2(pv[c + 2], pv[c + 3]),
                                   pack_bf16x2(pv[c + 4], pv[c + 5]), pack_bf16x2(pv[c + 6], pv[c + 7]));
        *reinterpret_cast<uint4*>(sm.dst + sw128(r, c, BLOCK_B)) = v;
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.ds_ready);
      // ---- dQ partial (lane = query row) -> fp32 atomics
      if (!mbar_wait_warp(&sm.dq_full, ph, p.status, kTimeoutAccFull)) { ok = false; break; }
      tc_fence_after();
      const int q = qt * BLOCK_B + r;
      float* dst = p.dq_acc + static_cast<size_t>(row0 + q) * (p.Hq * D) + static_cast<size_t>(h) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_addr + S_COL + c, rr);
        tmem_ld_wait();
        if (q < p.T) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            atomicAdd(reinterpret_cast<float4*>(dst + c) + i,
                      make_float4(__uint_as_float(rr[4 * i]), __uint_as_float(rr[4 * i + 1]),
                                  __uint_as_float(rr[4 * i + 2]), __uint_as_float(rr[4 * i + 3])));
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.dq_empty);
    }
    // ---- dK, dV (lane = key row) -> bf16
    if (ok && n_iter > 0 && mbar_wait_warp(&sm.dq_full, (n_iter - 1) & 1, p.status, kTimeoutAccFull)) {
      tc_fence_after();
      const bool key_ok = key < p.T;
      __nv_bfloat16* dkrow = p.dk + static_cast<size_t>(row0 + key) * p.ld_dk + p.dk_col0 + static_cast<size_t>(g) * D;
      __nv_bfloat16* dvrow = p.dv + static_cast<size_t>(row0 + key) * p.ld_dv + p.dv_col0 + static_cast<size_t>(g) * D;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = which == 0 ? DK_COL : DV_COL;
        __nv_bfloat16* out = which == 0 ? dkrow : dvrow;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
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
    } else if (n_iter == 0) {
      // No query can see these keys: their gradients are zero.
      if (key < p.T) {
        __nv_bfloat16* dkrow = p.dk + static_cast<size_t>(row0 + key) * p.ld_dk + p.dk_col0 + static_cast<size_t>(g) * D;
        __nv_bfloat16* dvrow = p.dv + static_cast<size_t>(row0 + key) * p.ld_dv + p.dv_col0 + static_cast<size_t>(g) * D;
        for (int c = 0; c < D; c += 8) {
          reinterpret_cast<uint4*>(dkrow + c)[0] = make_uint4(0, 0, 0, 0);
          reinterpret_cast<uint4*>(dvrow + c)[0] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// delta[b, h, t] = sum_d dO[t, h*D + d] * O[t, h*D + d]; one warp per (token, head).
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, int ld_o, const __nv_bfloat16* __restrict__ dout,
                                      int ld_do, float* __restrict__ delta, int B, int T, int Hq, int D) {
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(B) * T * Hq;
  if (wid >= total) return;
  const int h = static_cast<int>(wid % Hq);
  const long long tok = wid / Hq;
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
    const int b = static_cast<int>(tok / T), t = static_cast<int>(tok % T);
    delta[(static_cast<size_t>(b) * Hq + h) * T + t] = s;
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
//   dq_acc: fp32 scratch [B*T, Hq*D]; delta: fp32 scratch [B*Hq*T].
void attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
              int64_t q_col0, int64_t k_col0, int64_t v_col0, torch::Tensor lse, int64_t B, int64_t T, int64_t Hq,
              int64_t Hkv, int64_t D, torch::Tensor dq, int64_t dq_col0, torch::Tensor dk, int64_t dk_col0,
              torch::Tensor dv, int64_t dv_col0, torch::Tensor dq_acc, torch::Tensor delta, double scale,
              bool causal) {
  using namespace attn;
  for (auto* tp : {&q, &k, &v, &o, &dout, &dq, &dk, &dv}) check_cuda_bf16(*tp, "attn_bwd operand");
  TT_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TT_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TT_CHECK(dq_acc.scalar_type() == torch::kFloat32 && dq_acc.is_contiguous() && dq_acc.numel() >= B * T * Hq * D,
           "dq_acc must be fp32 [B*T, Hq*D]");
  TT_CHECK(delta.scalar_type() == torch::kFloat32 && delta.numel() >= B * Hq * T, "delta must be fp32 [B,Hq,T]");
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
  {
    const long long warps = tokens * Hq;
    attn_bwd_delta_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), static_cast<int>(o.stride(0)),
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), static_cast<int>(dout.stride(0)),
        delta.data_ptr<float>(), static_cast<int>(B), static_cast<int>(T), static_cast<int>(Hq), static_cast<int>(D));
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
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
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
  const CUtensorMap tq = attn_head_map(q), tk = attn_head_map(k), tv = attn_head_map(v), tdo = attn_head_map(dout);
  dim3 grid(static_cast<unsigned>((T + BLOCK_B - 1) / BLOCK_B), static_cast<unsigned>(Hkv), static_cast<unsigned>(B));
  if (D == 128) {
    const size_t smem = sizeof(BwdSmem<128>) + 1024;
    TT_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_bwd_kernel<128><<<grid, BWD_THREADS, smem, st>>>(tq, tk, tv, tdo, p);
  } else {
    const size_t smem = sizeof(BwdSmem<64>) + 1024;
    TT_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_bwd_kernel<64><<<grid, BWD_THREADS, smem, st>>>(tq, tk, tv, tdo, p);
  }
  TT_CUDA_CHECK(cudaGetLastError());
  const int width = static_cast<int>(Hq * D);
  const long long vecs = tokens * width / 8;
  attn_bwd_dq_convert_kernel<<<static_cast<unsigned>((vecs + 255) / 256), 256, 0, st>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), static_cast<int>(dq.stride(0)),
      static_cast<int>(dq_col0), tokens, width);
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
