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
// One CTA = one (batch, q head, 128-query tile).  Warp roles (192 threads):
//   warp 0: TMA producer (Q once; K/V tiles through a 2-deep ring)
//   warp 1: TMEM owner + MMA issuer: S = Q K^T into a double-buffered TMEM S,
//           O += P V into TMEM O (P from shared memory)
//   warps 2-5: softmax, one query row per thread (TMEM lane), online softmax in
//           fp32 with exp2; O is rescaled in TMEM only when the running row max
//           grows by more than 2^8 (otherwise the stale max is kept, which is
//           exact because the final normalisation uses the same reference max).
#include "common/host_utils.h"
#include "common/ptx.cuh"

namespace tt {
namespace attn {

constexpr int BLOCK = 128;
constexpr int THREADS = 192;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

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
};

template <int D>
struct FwdSmem {
  static constexpr int TILE_BYTES = BLOCK * D * 2;
  alignas(1024) uint8_t q[TILE_BYTES];
  alignas(1024) uint8_t k[2][TILE_BYTES];
  alignas(1024) uint8_t v[2][TILE_BYTES];
  alignas(1024) uint8_t p[BLOCK * BLOCK * 2];
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full, pv_done, done;
  uint32_t tmem_slot;
};

// Byte offset of element (row, col) inside a [rows][ncols] K-major bf16 tile stored as
// (ncols/64) chunks of [rows][128 B] with the 128-byte swizzle (matches TMA SWIZZLE_128B).
__device__ __forceinline__ uint32_t sw128_offset(int row, int col, int rows) {
  const int chunk = col >> 6;
  const int unit = (col & 63) >> 3;
  return static_cast<uint32_t>(chunk * rows * 128 + row * 128 + ((unit ^ (row & 7)) << 4) + ((col & 7) << 1));
}

template <int D>
__global__ void __launch_bounds__(THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  constexpr uint32_t TILE_BYTES = FwdSmem<D>::TILE_BYTES;
  constexpr uint32_t IDESC_QK = idesc_bf16_f32(BLOCK, BLOCK, false, false);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(BLOCK, D, false, true);
  constexpr uint32_t S_COL[2] = {0, BLOCK};
  constexpr uint32_t O_COL = 2 * BLOCK;
  constexpr uint32_t TMEM_COLS = 512;

  extern __shared__ uint8_t smem_raw[];
  FwdSmem<D>& sm = *reinterpret_cast<FwdSmem<D>*>(align_ptr(smem_raw, 1024));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_qt = (p.T + BLOCK - 1) / BLOCK;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // heaviest tiles first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int g = h / (p.Hq / p.Hkv);
  const int q_row0 = b * p.T + qt * BLOCK;
  const int k_row0 = b * p.Tk;
  const int n_kt_all = (p.Tk + BLOCK - 1) / BLOCK;
  int n_kt = n_kt_all;
  if (p.causal) {
    const int last_q = min(qt * BLOCK + BLOCK - 1, p.T - 1) + p.causal_offset;
    n_kt = min(n_kt_all, last_q / BLOCK + 1);
  }

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
      mbar_init(&sm.s_empty[i], 128);
    }
    mbar_init(&sm.p_full, 128);
    mbar_init(&sm.pv_done, 1);
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
    if (lane == 0 && n_kt > 0) {
      // ------------------------------------------------ producer
      mbar_arrive_expect_tx(&sm.q_full, TILE_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        tma_load_2d(sm.q + c * BLOCK * 128, &tmQ, &sm.q_full, p.q_col0 + h * D + c * 64, q_row0);
      for (int j = 0; j < n_kt; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&sm.k_empty[s], ph ^ 1u, p.status, kTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.k_full[s], TILE_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(sm.k[s] + c * BLOCK * 128, &tmK, &sm.k_full[s], p.k_col0 + g * D + c * 64,
                      k_row0 + j * BLOCK);
        if (!mbar_wait(&sm.v_empty[s], ph ^ 1u, p.status, kTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.v_full[s], TILE_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(sm.v[s] + c * BLOCK * 128, &tmV, &sm.v_full[s], p.v_col0 + g * D + c * 64,
                      k_row0 + j * BLOCK);
      }
      // Let every issued copy land before the CTA can exit.
      mbar_wait(&sm.q_full, 0, p.status, kTimeoutOther);
      for (int j = max(0, n_kt - 2); j < n_kt; ++j) {
        mbar_wait(&sm.k_full[j & 1], (j >> 1) & 1, p.status, kTimeoutOther);
        mbar_wait(&sm.v_full[j & 1], (j >> 1) & 1, p.status, kTimeoutOther);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_kt > 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t q_base = smem_u32(sm.q);
      const uint32_t p_base = smem_u32(sm.p);
      bool ok = mbar_wait(&sm.q_full, 0, p.status, kTimeoutFull);
      auto issue_qk = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&sm.s_empty[s], ph ^ 1u, p.status, kTimeoutAccEmpty)) return false;
        if (!mbar_wait(&sm.k_full[s], ph, p.status, kTimeoutFull)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sm.k[s]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BLOCK * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + S_COL[s], sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024),
                      IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&sm.k_empty[s]);
        umma_commit(&sm.s_full[s]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; ok && j < n_kt; ++j) {
        if (j + 1 < n_kt && !issue_qk(j + 1)) break;
        const int s = j & 1;
        if (!mbar_wait(&sm.p_full, j & 1, p.status, kTimeoutFull)) break;
        if (!mbar_wait(&sm.v_full[s], (j >> 1) & 1, p.status, kTimeoutFull)) break;
        tc_fence_after();
        const uint32_t v_base = smem_u32(sm.v[s]);
#pragma unroll
        for (int kk = 0; kk < BLOCK / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * (BLOCK * 128) + (kk & 3) * 32;
          const uint32_t b_off = kk * 16 * 128;
          umma_f16_ss(tmem + O_COL, sdesc_sw128(p_base + a_off, 16, 1024),
                      sdesc_sw128(v_base + b_off, BLOCK * 128, 1024), IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&sm.v_empty[s]);
        umma_commit(&sm.pv_done);
      }
      umma_commit(&sm.done);
      mbar_wait(&sm.done, 0, p.status, kTimeoutOther);
    }
  } else {
    // ------------------------------------------------ softmax (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                 // query row within the tile == TMEM lane
    const int q_idx = qt * BLOCK + r;                  // query position within the sequence
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int q_lim = q_idx + p.causal_offset;          // last key this row may attend (causal)
    float m_ref = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const int s = j & 1;
      if (!mbar_wait_warp(&sm.s_full[s], (j >> 1) & 1, p.status, kTimeoutAccFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[BLOCK];
#pragma unroll
      for (int c = 0; c < BLOCK; c += 32) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_addr + S_COL[s] + c, rr);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c + i] = __uint_as_float(rr[i]);
      }
      tc_fence_before();
      mbar_arrive(&sm.s_empty[s]);
      // mask + scale into log2 domain
      const int key0 = j * BLOCK;
      const bool need_mask = (key0 + BLOCK > p.Tk) || (p.causal && key0 + BLOCK - 1 > q_lim);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < BLOCK; ++i) {
        float x = sv[i] * p.scale_log2;
        if (need_mask) {
          const int key = key0 + i;
          if (key >= p.Tk || (p.causal && key > q_lim)) x = -INFINITY;
        }
        sv[i] = x;
        mx = fmaxf(mx, x);
      }
      float alpha = 1.0f;
      bool rescale = false;
      if (mx > m_ref + RESCALE_THRESHOLD || (m_ref == -INFINITY && mx != -INFINITY)) {
        alpha = (m_ref == -INFINITY) ? 0.0f : exp2f(m_ref - mx);
        rescale = (j > 0);
        m_ref = mx;
      }
      const float mref = (m_ref == -INFINITY) ? 0.0f : m_ref;
      float rs = 0.0f;
#pragma unroll
      for (int i = 0; i < BLOCK; ++i) {
        const float e = exp2f(sv[i] - mref);
        sv[i] = e;
        rs += e;
      }
      l = l * alpha + rs;
      // P buffer and O are free once the previous PV MMA retired.
      if (j > 0) {
        if (!mbar_wait_warp(&sm.pv_done, (j - 1) & 1, p.status, kTimeoutAccFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // tcgen05.ld/st are warp-collective: if any lane of the warp must rescale its O row,
      // the whole warp runs the loop (alpha == 1 for rows that did not change).
      if (__any_sync(0xffffffffu, rescale)) {
        if (!rescale) alpha = 1.0f;
#pragma unroll
        for (int c = 0; c < D; c += 16) {
          uint32_t ov[16];
          tmem_ld16(tmem + lane_addr + O_COL + c, ov);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st16(tmem + lane_addr + O_COL + c, ov);
        }
        tmem_st_wait();
      }
      // P row -> shared memory (bf16, K-major, 128B swizzle)
#pragma unroll
      for (int c = 0; c < BLOCK; c += 8) {
        const uint4 v = make_uint4(pack_bf16x2(sv[c], sv[c + 1]), pack_bf16x2(sv[c + 2], sv[c + 3]),
                                   pack_bf16x2(sv[c + 4], sv[c + 5]), pack_bf16x2(sv[c + 6], sv[c + 7]));
        *reinterpret_cast<uint4*>(sm.p + sw128_offset(r, c, BLOCK)) = v;
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.p_full);
    }
    // ------------------------------------------------ epilogue: O / l, LSE
    if (ok && n_kt > 0 && mbar_wait_warp(&sm.pv_done, (n_kt - 1) & 1, p.status, kTimeoutAccFull)) {
      tc_fence_after();
      const float inv_l = (l > 0.0f) ? 1.0f / l : 0.0f;
      const bool row_ok = q_idx < p.T;
      __nv_bfloat16* orow = p.o + static_cast<size_t>(q_row0 + r) * p.ld_o + static_cast<size_t>(h) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t ov[32];
        tmem_ld32(tmem + lane_addr + O_COL + c, ov);
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
  const CUtensorMap tq = head_map(q), tk = head_map(k), tv = head_map(v);
  dim3 grid(static_cast<unsigned>((T + BLOCK - 1) / BLOCK), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  if (D == 128) {
    const size_t smem = sizeof(FwdSmem<128>) + 1024;
    TT_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_fwd_kernel<128><<<grid, THREADS, smem, cur_stream()>>>(tq, tk, tv, p);
  } else {
    const size_t smem = sizeof(FwdSmem<64>) + 1024;
    TT_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attn_fwd_kernel<64><<<grid, THREADS, smem, cur_stream()>>>(tq, tk, tv, p);
  }
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
