// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-gen tensor cores.
//
//   C[M,N] = alpha * sum_k A(m,k) * B(n,k)      (fp32 accumulate in TMEM)
//
// Operands are staged by TMA (tiled, 128-byte swizzle, one CTA per load, local
// memory only) into a STAGES-deep shared-memory ring; one elected thread issues
// tcgen05.mma (kind::f16, M=128, N=BN, K=16) into a double-buffered TMEM
// accumulator; four epilogue warps drain TMEM with tcgen05.ld and apply the
// epilogue while the next tile's MMAs run.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +31).
//
// Either operand may be K-major (row-major [rows, K]) or MN-major (row-major
// [K, rows]); that covers y = x W^T (fwd), dx = dy W (dgrad) and dW = dy^T x
// (wgrad) without transposes.  Epilogues: bf16 store, fp32 store, fp32
// accumulate (gradient accumulation into fp32 master grads), SwiGLU (gate|up
// weight halves fused into one 256-wide tile, writes silu(g)*u and optionally
// g|u for backward), and SwiGLU-backward (dact -> d[g|u]).
//
// Grouped mode (MoE experts): the token operand's rows are grouped by expert in
// segments [grp_off[e], grp_off[e+1]) that start on multiples of 128 (padding rows
// are zero).  GROUP_M: C_rows = A_rows B_e^T with each 128-row tile's expert found
// from grp_off (forward and dgrad); GROUP_K: C_e (+)= A_e^T B_e with the reduction
// running over expert e's token segment only (weight gradients).  grp_off lives on
// the device, so routing never synchronises with the host.
//
// Replaces the reference's nn.Linear/cuBLAS projections
// (tinytron/model/modules/attn.py:141-145, mlp.py:27-29,45, gpt.py:60,109) and the
// SiLU*up elementwise op (mlp.py:45); grouped mode replaces the expert GEMMs
// (F.grouped_mm / bmm, mlp.py:157-187).
#include "common/ptx.cuh"
#include "common/host_utils.h"

#include <atomic>
#include <cstdlib>

namespace tt {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int NUM_THREADS = 192;

// EPI_AXPBY: bf16 out = alpha * acc + beta * aux (a bf16 [M, N] addend), the fused
// "a*X + B@X" / "b*A + c*A@A" steps of the Newton-Schulz iteration.
enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_F32_ACC = 2, EPI_SWIGLU = 3, EPI_DSWIGLU = 4, EPI_AXPBY = 5 };
// GROUP_SYM: the output is symmetric (C = X X^T, or A A^T with A symmetric); only the
// 128x128 tiles on or above the diagonal are computed, and each off-diagonal tile is
// also stored transposed into its mirror position.  GROUP_SYM and GROUP_BATCH run
// n_groups independent products of one shape stacked along the rows (batch g reads A
// rows from g * a_grp_rows, B rows / K coordinates from g * b_grp_rows, and writes C and
// reads the addend at rows g * c_grp_rows): one launch for a whole set of matrices.
enum Group : int { GROUP_NONE = 0, GROUP_M = 1, GROUP_K = 2, GROUP_SYM = 3, GROUP_BATCH = 4 };

template <int GROUP>
constexpr bool kBatched = (GROUP == GROUP_SYM || GROUP == GROUP_BATCH);

struct Params {
  int M, N, K;                 // output rows, output cols, reduction length
  void* C;                     // output (bf16 or fp32), row stride ldc elements
  int ldc;
  const __nv_bfloat16* aux;    // DSWIGLU: g|u pre-activations [M, 2N]
  int ld_aux;
  __nv_bfloat16* aux_out;      // SWIGLU: optional g|u store [M, 2N]; DSWIGLU: d(g|u) [M, 2N]
  int ld_aux_out;
  float alpha;
  float beta;                  // EPI_AXPBY: weight of the addend `aux`
  const float* alpha_ptr;      // optional device scalar multiplied into alpha
  int b_row_offset2;           // SWIGLU: first row of the "up" half inside B
  int* status;                 // device status word for bounded waits
  // Grouped mode only.
  const int* grp_off;          // [n_groups + 1] segment starts (multiples of BM), device
  int n_groups;
  int b_grp_rows;              // GROUP_M: per-group offset of B rows (K-major) or K coordinate (MN-major)
  int b_split_kb;              // GROUP_M, MN-major B: k-blocks >= this come from rows b_off2 + ...
  int b_off2;
  int c_grp_rows;              // GROUP_K, batched modes: per-group row offset of C (and of the addend)
  int a_grp_rows;              // batched modes: per-group row offset of A
  // CTA-pair kernel, fp32-accumulate epilogue only: the reduction is split into split_k
  // ranges whose epilogues add into C one after another (split s waits until the 16
  // epilogue warps of split s-1 counted themselves in splitk_flags[tile]), so the sum
  // order is fixed and results are deterministic.
  int split_k;
  int* splitk_flags;
  // bf16 epilogue only: when set, output row r goes to the address row_ptr[r] (0: row
  // dropped) instead of C + r * ldc.  The expert-parallel combine uses it to store each
  // expert output row straight into the memory of the rank that owns the token (a peer
  // address over NVLink), so the transfer overlaps the GEMM tile by tile.
  const long long* row_ptr;
};

struct TileInfo {
  int mb, nb;  // tile coordinates (rows of A / C, columns of C)
  int grp;     // group (expert) of the tile
  int kb0;     // first k-block (GROUP_K: start of the group's token segment)
  int nk;      // number of k-blocks (GROUP_K: 0 for an empty group -> tile skipped)
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  // Grouped order: 16 M-blocks share each sweep over N, so concurrently running
  // CTAs reuse both A rows and B rows from L2.
  constexpr int GROUP = 16;
  const int group_tiles = GROUP * num_n;
  const int g = tile / group_tiles;
  const int first_m = g * GROUP;
  const int gm = min(num_m - first_m, GROUP);
  const int in = tile - g * group_tiles;
  mb = first_m + in % gm;
  nb = in / gm;
}

template <int GROUP>
__device__ __forceinline__ TileInfo decode_tile(int tile, int num_m, int num_n, int num_k, const Params& p) {
  TileInfo t;
  t.grp = 0;
  t.kb0 = 0;
  t.nk = num_k;
  if constexpr (GROUP == GROUP_SYM) {  // row-major walk over the upper triangle (num_m == num_n)
    const int per = num_m * (num_m + 1) / 2;
    t.grp = tile / per;
    int mb = 0, rem = tile - t.grp * per;
    while (rem >= num_m - mb) {
      rem -= num_m - mb;
      ++mb;
    }
    t.mb = mb;
    t.nb = mb + rem;
  } else if constexpr (GROUP == GROUP_BATCH) {
    const int per = num_m * num_n;
    t.grp = tile / per;
    tile_coords(tile - t.grp * per, num_m, num_n, t.mb, t.nb);
  } else if constexpr (GROUP == GROUP_K) {
    const int per = num_m * num_n;
    t.grp = tile / per;
    tile_coords(tile - t.grp * per, num_m, num_n, t.mb, t.nb);
    const int r0 = __ldg(p.grp_off + t.grp), r1 = __ldg(p.grp_off + t.grp + 1);
    t.kb0 = r0 / BK;
    t.nk = (r1 - r0) / BK;
  } else {
    tile_coords(tile, num_m, num_n, t.mb, t.nb);
    if constexpr (GROUP == GROUP_M) {  // last group starting at or before the tile's first row
      const int row = t.mb * BM;
      int lo = 0, hi = p.n_groups - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(p.grp_off + mid) <= row) lo = mid;
        else hi = mid - 1;
      }
      t.grp = lo;
    }
  }
  return t;
}

// Logistic sigmoid with the approximate exponential and the approximate division
// (__fdividef): two special-function ops and a few FMAs, against a branchy IEEE-exact
// division sequence per element; the results are rounded to bf16 afterwards.  For x below
// about -88 the exponential overflows to inf and __fdividef(1, inf) gives 0, the limit.
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Store n (<= 32) fp32 values as bf16 starting at dst; vectorised when a full aligned run.
template <int NV>
__device__ __forceinline__ void store_bf16(__nv_bfloat16* dst, const float (&v)[NV], int n_valid) {
  if (n_valid >= NV) {
    uint32_t packed[NV / 2];
#pragma unroll
    for (int i = 0; i < NV / 2; ++i) packed[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < NV / 8; ++i)
      d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i)
      if (i < n_valid) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

template <int NV>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* src, float (&v)[NV], int n_valid) {
  if (n_valid >= NV) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < NV / 8; ++i) {
      uint4 q = s4[i];
      float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y), c = unpack_bf16x2(q.z), d = unpack_bf16x2(q.w);
      v[8 * i + 0] = a.x; v[8 * i + 1] = a.y; v[8 * i + 2] = b.x; v[8 * i + 3] = b.y;
      v[8 * i + 4] = c.x; v[8 * i + 5] = c.y; v[8 * i + 6] = d.x; v[8 * i + 7] = d.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = (i < n_valid) ? __bfloat162float(src[i]) : 0.0f;
  }
}

// Epilogue of one 128-row accumulator slice: thread = one TMEM lane = one output row.
// Drains BN fp32 columns from TMEM (t_row) and applies EPI; nb is the tile's column block.
template <int BN, int EPI>
// [c_lo, c_hi): the slice of output columns of the tile this thread handles (the CTA-pair
// kernel splits a row between two epilogue warpgroups); defaults cover the whole tile.
// `mirror` (GROUP_SYM, off-diagonal tiles): every stored value (row, col) is also stored
// at (col, row); lanes hold consecutive rows, so each mirrored column is one 64-byte
// warp-wide store.
// (the mirrored store of batch g goes to rows mirror_row0 + col, column mirror_col).
__device__ __forceinline__ void epilogue_row(const Params& p, uint32_t t_row, int nb, int row, bool row_ok,
                                             float alpha, int c_lo = 0, int c_hi = 1 << 30, bool mirror = false,
                                             int mirror_row0 = 0, int mirror_col = 0) {
  constexpr int OUT_BN = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  c_hi = min(c_hi, OUT_BN);
  if constexpr (EPI == EPI_F32_ACC) {
    // C (fp32) is read 64 columns at a time (16 independent 16-byte loads in flight per
    // thread) before the TMEM reads of those columns: the read-modify-write latency is
    // paid BN/64 times per tile, which matters for short-K tiles (MoE weight gradients).
    constexpr int QC = 64;
    float* crow = reinterpret_cast<float*>(p.C) + static_cast<size_t>(row) * p.ldc;
#pragma unroll 1
    for (int q0 = c_lo; q0 < c_hi; q0 += QC) {
      const int colq = nb * BN + q0;
      const bool full = row_ok && colq + QC <= p.N;
      float4 cq[QC / 4];
      if (full) {
#pragma unroll
        for (int i = 0; i < QC / 4; ++i) cq[i] = reinterpret_cast<const float4*>(crow + colq)[i];
      }
#pragma unroll
      for (int c = 0; c < QC; c += 32) {
        uint32_t r[32];
        tmem_ld32(t_row + q0 + c, r);
        tmem_ld_wait();
        const int col0 = colq + c;
        if (full) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 o = cq[c / 4 + i];
            reinterpret_cast<float4*>(crow + col0)[i] =
                make_float4(o.x + __uint_as_float(r[4 * i]) * alpha, o.y + __uint_as_float(r[4 * i + 1]) * alpha,
                            o.z + __uint_as_float(r[4 * i + 2]) * alpha, o.w + __uint_as_float(r[4 * i + 3]) * alpha);
          }
        } else if (row_ok && col0 < p.N) {
          const int nv = min(32, p.N - col0);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nv) crow[col0 + i] += __uint_as_float(r[i]) * alpha;
        }
      }
    }
  } else if constexpr (EPI == EPI_BF16 || EPI == EPI_F32 || EPI == EPI_AXPBY) {
    __nv_bfloat16* brow = nullptr;
    if constexpr (EPI == EPI_BF16 || EPI == EPI_AXPBY) {
      if (p.row_ptr != nullptr) {
        const long long a = row_ok ? p.row_ptr[row] : 0ll;
        brow = reinterpret_cast<__nv_bfloat16*>(a);
        row_ok = row_ok && a != 0ll;
      } else {
        brow = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<size_t>(row) * p.ldc;
      }
    }
#pragma unroll 1
    for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(t_row + c0, r);
      tmem_ld_wait();
      const int col0 = nb * BN + c0;
      if (row_ok && col0 < p.N) {
        const int nv = min(32, p.N - col0);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * alpha;
        if constexpr (EPI == EPI_AXPBY) {
          float av[32];
          load_bf16<32>(p.aux + static_cast<size_t>(row) * p.ld_aux + col0, av, nv);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaf(p.beta, av[i], v[i]);
        }
        if constexpr (EPI == EPI_BF16 || EPI == EPI_AXPBY) {
          store_bf16<32>(brow + col0, v, nv);
          if (mirror) {
            __nv_bfloat16* cb = reinterpret_cast<__nv_bfloat16*>(p.C);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nv)
                cb[static_cast<size_t>(mirror_row0 + col0 + i) * p.ldc + mirror_col] = __float2bfloat16_rn(v[i]);
          }
        } else {
          float* dst = reinterpret_cast<float*>(p.C) + static_cast<size_t>(row) * p.ldc + col0;
          if (nv == 32) {
            float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
              if constexpr (EPI == EPI_F32_ACC) {
                const float4 c = d4[i];
                o.x += c.x; o.y += c.y; o.z += c.z; o.w += c.w;
              }
              d4[i] = o;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i < nv) {
                if constexpr (EPI == EPI_F32_ACC) dst[i] += v[i];
                else dst[i] = v[i];
              }
            }
          }
        }
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
    for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
      uint32_t g[16], u[16];
      tmem_ld16(t_row + c0, g);
      tmem_ld16(t_row + OUT_BN + c0, u);
      tmem_ld_wait();
      const int col0 = nb * OUT_BN + c0;
      if (row_ok && col0 < p.N) {
        const int nv = min(16, p.N - col0);
        float gv[16], uv[16], o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          gv[i] = __uint_as_float(g[i]);
          uv[i] = __uint_as_float(u[i]);
          o[i] = silu_f(gv[i]) * uv[i];
        }
        store_bf16<16>(reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<size_t>(row) * p.ldc + col0, o, nv);
        if (p.aux_out != nullptr) {
          __nv_bfloat16* base = p.aux_out + static_cast<size_t>(row) * p.ld_aux_out;
          store_bf16<16>(base + col0, gv, nv);
          store_bf16<16>(base + p.N + col0, uv, nv);
        }
      }
    }
  } else if constexpr (EPI == EPI_DSWIGLU) {
    // The saved pre-activations g|u are read 32 columns at a time (8 independent 16-byte
    // loads per thread), double-buffered: the loads of the next 32 columns are issued
    // before the current ones are processed, so the load latency is paid once per row
    // segment instead of once per block.
    constexpr int QC = 32;
    const __nv_bfloat16* a = p.aux + static_cast<size_t>(row) * p.ld_aux;
    __nv_bfloat16* o = p.aux_out + static_cast<size_t>(row) * p.ld_aux_out;
    uint4 gA[QC / 8], uA[QC / 8], gB[QC / 8], uB[QC / 8];
    auto fetch = [&](int q0, uint4(&gq)[QC / 8], uint4(&uq)[QC / 8]) {
      const int colq = nb * BN + q0;
      if (row_ok && colq + QC <= p.N) {
#pragma unroll
        for (int i = 0; i < QC / 8; ++i) {
          gq[i] = __ldg(reinterpret_cast<const uint4*>(a + colq) + i);
          uq[i] = __ldg(reinterpret_cast<const uint4*>(a + p.N + colq) + i);
        }
      }
    };
    auto process = [&](int q0, const uint4(&gq)[QC / 8], const uint4(&uq)[QC / 8]) {
      const int colq = nb * BN + q0;
      const bool full = row_ok && colq + QC <= p.N;
#pragma unroll
      for (int c = 0; c < QC; c += 16) {
        uint32_t r[16];
        tmem_ld16(t_row + q0 + c, r);
        tmem_ld_wait();
        const int col0 = colq + c;
        if (row_ok && col0 < p.N) {
          const int nv = min(16, p.N - col0);
          float gv[16], uv[16], dg[16], du[16];
          if (full) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gq[c / 8 + h]);
              const uint32_t* uw = reinterpret_cast<const uint32_t*>(&uq[c / 8 + h]);
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const float2 gf = unpack_bf16x2(gw[w]), uf = unpack_bf16x2(uw[w]);
                gv[8 * h + 2 * w] = gf.x;
                gv[8 * h + 2 * w + 1] = gf.y;
                uv[8 * h + 2 * w] = uf.x;
                uv[8 * h + 2 * w + 1] = uf.y;
              }
            }
          } else {
            load_bf16<16>(a + col0, gv, nv);
            load_bf16<16>(a + p.N + col0, uv, nv);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float d = __uint_as_float(r[i]) * alpha;
            const float sg = sigmoid_f(gv[i]);
            du[i] = d * gv[i] * sg;
            dg[i] = d * uv[i] * sg * (1.0f + gv[i] * (1.0f - sg));
          }
          store_bf16<16>(o + col0, dg, nv);
          store_bf16<16>(o + p.N + col0, du, nv);
        }
      }
    };
    // (c_hi - c_lo) is a multiple of 2 * QC for every caller (128 or 256 columns).
    fetch(c_lo, gA, uA);
#pragma unroll 1
    for (int q0 = c_lo; q0 < c_hi; q0 += 2 * QC) {
      fetch(q0 + QC, gB, uB);
      process(q0, gA, uA);
      if (q0 + 2 * QC < c_hi) fetch(q0 + 2 * QC, gA, uA);
      process(q0 + QC, gB, uB);
    }
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, int GROUP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, A_MN, B_MN);
  constexpr int OUT_BN = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  static_assert(BN == 128 || BN == 256, "BN must be 128 or 256");
  static_assert(EPI != EPI_SWIGLU || (BN == 256 && !B_MN), "SwiGLU epilogue needs BN=256, K-major B");
  static_assert(GROUP != GROUP_K || (A_MN && B_MN), "GROUP_K reduces over token rows: both operands MN-major");
  static_assert(GROUP != GROUP_M || !A_MN, "GROUP_M: A holds the grouped token rows, K-major");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_ptr(smem_raw, 1024);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // GROUP_M: the row count is the padded token total, known only on the device.
  const int M = (GROUP == GROUP_M) ? __ldg(p.grp_off + p.n_groups) : p.M;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (p.N + OUT_BN - 1) / OUT_BN;
  const int num_tiles = (GROUP == GROUP_SYM) ? num_m * (num_m + 1) / 2 * p.n_groups
                                             : num_m * num_n * ((GROUP == GROUP_K || GROUP == GROUP_BATCH) ? p.n_groups : 1);
  const int num_k = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(done_bar, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pending = 0;        // bit s: stage s has an issued load
      uint32_t pending_phase = 0;  // bit s: parity of that load's fill
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const TileInfo t = decode_tile<GROUP>(tile, num_m, num_n, num_k, p);
        const int mb = t.mb, nb = t.nb;
        const int b_rows0 = (GROUP == GROUP_M || kBatched<GROUP>) ? t.grp * p.b_grp_rows : 0;
        const int a_rows0 = kBatched<GROUP> ? t.grp * p.a_grp_rows : 0;
        for (int kb = 0; kb < t.nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int kc = (t.kb0 + kb) * BK;  // k coordinate (token row for GROUP_K)
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], kc, a_rows0 + mb * BM);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_2d(a_dst + c * (BK * 128), &tmA, &full[stage], mb * BM + c * 64, kc);
          }
          if constexpr (EPI == EPI_SWIGLU) {
            tma_load_2d(b_dst, &tmB, &full[stage], kc, b_rows0 + nb * (BN / 2));
            tma_load_2d(b_dst + (BN / 2) * 128, &tmB, &full[stage], kc, p.b_row_offset2 + b_rows0 + nb * (BN / 2));
          } else if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full[stage], kc, b_rows0 + nb * BN);
          } else {
            int kb_b = kc;
            if constexpr (GROUP == GROUP_M)
              kb_b = (kb < p.b_split_kb) ? b_rows0 + kb * BK : p.b_off2 + b_rows0 + (kb - p.b_split_kb) * BK;
            if constexpr (kBatched<GROUP>) kb_b = b_rows0 + kc;
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(b_dst + c * (BK * 128), &tmB, &full[stage], nb * BN + c * 64, kb_b);
          }
          pending |= (1u << stage);
          pending_phase = (pending_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Wait (bounded) until every load this thread issued has landed, so no
      // copy is still writing shared memory when the CTA exits.
      for (int s = 0; s < STAGES; ++s)
        if (pending & (1u << s)) mbar_wait(&full[s], (pending_phase >> s) & 1u, p.status, kTimeoutOther);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int nk = decode_tile<GROUP>(tile, num_m, num_n, num_k, p).nk;
        if (nk == 0) continue;  // empty group (GROUP_K): no accumulator used
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, p.status, kTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_base + j * 2048, BK * 128, 1024)
                                     : sdesc_sw128(a_base + j * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_base + j * 2048, BK * 128, 1024)
                                     : sdesc_sw128(b_base + j * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, IDESC, (kb > 0 || j > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);  // stage is free once these MMAs retire
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);  // accumulator ready once the tile's MMAs retire
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: every MMA issued above must retire before TMEM is released.
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, p.status, kTimeoutOther);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    float alpha = p.alpha;
    if (p.alpha_ptr != nullptr) alpha *= *p.alpha_ptr;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const TileInfo t = decode_tile<GROUP>(tile, num_m, num_n, num_k, p);
      if (t.nk == 0) continue;
      const int nb = t.nb;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, p.status, kTimeoutAccFull)) break;
      tc_fence_after();
      const int row_local = t.mb * BM + row_in_tile;
      const bool row_ok = row_local < M;
      const int row = (GROUP == GROUP_K || kBatched<GROUP>) ? t.grp * p.c_grp_rows + row_local : row_local;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);

      epilogue_row<BN, EPI>(p, t_row, nb, row, row_ok, alpha, 0, 1 << 30, GROUP == GROUP_SYM && t.mb != t.nb,
                            t.grp * p.c_grp_rows, row_local);
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ---------------------------------------------------------------------------- CTA-pair kernel
// 256 x 256 output tiles computed by a cluster of two CTAs with cta_group::2 MMAs
// (M = 256, N = 256, K = 16 per instruction).  CTA r of the pair loads A rows
// [256*mb + 128*r, +128) and B rows [256*nb + 128*r, +128) (SwiGLU: CTA 0 the gate rows,
// CTA 1 the up rows of column block nb) into its own shared memory with plain TMA loads
// that both signal the even CTA's `full` barrier; the even CTA's single MMA thread issues
// the pair MMAs, and tcgen05.commit multicasts stage-free and accumulator-ready to both
// CTAs.  Each CTA's TMEM holds its 128 rows x 256 columns (two buffers); its four
// epilogue warps drain them with the same epilogues as the single-CTA kernel and release
// the buffer on the even CTA's barrier.  Per CTA and k-block the pair moves 32 KB of
// operands for 512 MMA cycles (the single-CTA 128 x 256 tile moves 48 KB), so the
// operand traffic per flop drops by a third.
constexpr int BN2 = 256;
constexpr int STAGES2 = 6;
constexpr int PAIR_THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue (two warpgroups)
constexpr uint32_t PAIR_A_BYTES = BM * BK * 2;
constexpr uint32_t PAIR_B_BYTES = 128 * BK * 2;

// Grouped mode (GROUP_M, MoE experts): the token rows are laid out in expert segments
// that start on multiples of 256 (so a pair tile never straddles two experts); the tile's
// expert selects B's rows (K-major) or K offset (MN-major) as in the single-CTA kernel.
template <int GROUP>
__device__ __forceinline__ int pair_tile_group(const Params& p, int mb) {
  if constexpr (GROUP != GROUP_M) {
    return 0;
  } else {
    const int row = mb * 256;
    int lo = 0, hi = p.n_groups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(p.grp_off + mid) <= row) lo = mid;
      else hi = mid - 1;
    }
    return lo;
  }
}

template <bool A_MN, bool B_MN, int EPI, int GROUP = GROUP_NONE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PAIR_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  constexpr uint32_t TMEM_COLS = 2 * BN2;
  constexpr uint32_t IDESC = idesc_bf16_f32(256, BN2, A_MN, B_MN);
  constexpr int OUT_BN = (EPI == EPI_SWIGLU) ? BN2 / 2 : BN2;
  static_assert(EPI != EPI_SWIGLU || !B_MN, "SwiGLU epilogue needs K-major B");
  static_assert(!kBatched<GROUP>, "batched and symmetric products run on the single-CTA kernel");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_ptr(smem_raw, 1024);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES2 * PAIR_A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES2 * PAIR_B_BYTES);
  uint64_t* empty = full + STAGES2;
  uint64_t* acc_full = empty + STAGES2;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  static_assert(GROUP != GROUP_K || (A_MN && B_MN && EPI == EPI_F32_ACC),
                "grouped-K (MoE weight gradients) reduces over token rows: MN-major operands, fp32 accumulate");
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int n_pairs = static_cast<int>(gridDim.x >> 1);
  // GROUP_M: the row count is the padded token total, known only on the device.
  const int M = (GROUP == GROUP_M) ? __ldg(p.grp_off + p.n_groups) : p.M;
  const int num_m = (M + 255) / 256;
  const int num_n = (p.N + OUT_BN - 1) / OUT_BN;
  // GROUP_K: one tile set per group (expert); the reduction runs over the group's token
  // segment [grp_off[g], grp_off[g+1]) and the output rows are offset by g * c_grp_rows.
  const int num_tiles = num_m * num_n * (GROUP == GROUP_K ? p.n_groups : 1);
  const int num_k = (p.K + BK - 1) / BK;
  const int S = (GROUP != GROUP_K && EPI == EPI_F32_ACC && p.split_k > 1) ? p.split_k : 1;
  const int num_units = num_tiles * S;
  const int kb_per = (num_k + S - 1) / S;
  // (group, m block, n block, first k-block, end k-block) of a work unit; the three roles
  // derive it identically, so an empty group's tiles are skipped by all of them.
  auto unit_info = [&](int unit, int& grp, int& mb, int& nb, int& kb_lo, int& kb_hi) {
    const int tile = unit / S, split = unit - (unit / S) * S;
    if constexpr (GROUP == GROUP_K) {
      const int per = num_m * num_n;
      grp = tile / per;
      tile_coords(tile - grp * per, num_m, num_n, mb, nb);
      kb_lo = __ldg(p.grp_off + grp) / BK;
      kb_hi = __ldg(p.grp_off + grp + 1) / BK;
    } else {
      grp = 0;
      tile_coords(tile, num_m, num_n, mb, nb);
      kb_lo = split * kb_per;
      kb_hi = min(num_k, (split + 1) * kb_per);
    }
  };

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 16);  // one arrival per epilogue warp, 8 warps x 2 CTAs
    }
    mbar_init(done_bar, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      const uint32_t full0 = mapa_shared(smem_u32(&full[0]), 0);  // the even CTA's full[0]
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = pair; ok && unit < num_units; unit += n_pairs) {
        int grp, mb, nb, kb_lo, kb_hi;
        unit_info(unit, grp, mb, nb, kb_lo, kb_hi);
        const int grp_rows = (GROUP == GROUP_M) ? pair_tile_group<GROUP>(p, mb) * p.b_grp_rows : 0;
        const int a_row0 = mb * 256 + static_cast<int>(crank) * 128;
        // K-major B: first B row of this CTA's half; MN-major B: first N column of it.
        const int b_row0 = (EPI == EPI_SWIGLU) ? (crank ? p.b_row_offset2 : 0) + grp_rows + nb * 128
                           : (B_MN ? nb * BN2 + static_cast<int>(crank) * 128
                                   : grp_rows + nb * BN2 + static_cast<int>(crank) * 128);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, p.status, kTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (PAIR_A_BYTES + PAIR_B_BYTES));
          const uint32_t bar = full0 + static_cast<uint32_t>(stage) * 8u;
          uint8_t* a_dst = sA + stage * PAIR_A_BYTES;
          uint8_t* b_dst = sB + stage * PAIR_B_BYTES;
          const int kc = kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, bar, kc, a_row0);
          } else {
#pragma unroll
            for (int c = 0; c < 2; ++c) tma_load_2d_pair(a_dst + c * (BK * 128), &tmA, bar, a_row0 + c * 64, kc);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, bar, kc, b_row0);
          } else {
            int kb_b = kc;
            if constexpr (GROUP == GROUP_M)
              kb_b = (kb < p.b_split_kb) ? grp_rows + kb * BK : p.b_off2 + grp_rows + (kb - p.b_split_kb) * BK;
#pragma unroll
            for (int c = 0; c < 2; ++c) tma_load_2d_pair(b_dst + c * (BK * 128), &tmB, bar, b_row0 + c * 64, kb_b);
          }
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------ MMA issuer (even CTA only)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int unit = pair; ok && unit < num_units; unit += n_pairs) {
        int grp, mb, nb, kb0, kb_end;
        unit_info(unit, grp, mb, nb, kb0, kb_end);
        if (GROUP == GROUP_K && kb_end <= kb0) continue;  // empty group: no accumulator used
        if (!mbar_wait_cluster(&acc_empty[acc], acc_phase ^ 1u, p.status, kTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN2);
        for (int kb = kb0; kb < kb_end; ++kb) {
          if (!mbar_wait_cluster(&full[stage], phase, p.status, kTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * PAIR_A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * PAIR_B_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_base + j * 2048, BK * 128, 1024)
                                     : sdesc_sw128(a_base + j * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_base + j * 2048, BK * 128, 1024)
                                     : sdesc_sw128(b_base + j * 32, 16, 1024);
            umma_f16_ss_pair(d_tmem, ad, bd, IDESC, (kb > kb0 || j > 0) ? 1u : 0u);
          }
          umma_commit_pair_mc(&empty[stage], 0x3);  // stage free in both CTAs
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(&acc_full[acc], 0x3);  // accumulator ready in both CTAs
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit_pair(done_bar);
      mbar_wait(done_bar, 0, p.status, kTimeoutOther);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..9, both CTAs)
    // Warp w reads TMEM lanes 32*(w%4)..+31; warps 2..5 take the tile's first half of the
    // output columns and warps 6..9 the second, so two warps drain each row.
    const int q = warp & 3;
    const int col_half = (warp - 2) >> 2;
    constexpr int OUT_BN_T = (EPI == EPI_SWIGLU) ? BN2 / 2 : BN2;
    float alpha = p.alpha;
    if (p.alpha_ptr != nullptr) alpha *= *p.alpha_ptr;
    const uint32_t acc_empty0_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int unit = pair; ok && unit < num_units; unit += n_pairs) {
      const int tile = unit / S, split = unit - (unit / S) * S;
      int grp, mb, nb, kb_lo, kb_hi;
      unit_info(unit, grp, mb, nb, kb_lo, kb_hi);
      if (GROUP == GROUP_K && kb_hi <= kb_lo) continue;  // empty group: nothing was accumulated
      if (!mbar_wait_cluster_warp(&acc_full[acc], acc_phase, p.status, kTimeoutAccFull)) break;
      tc_fence_after();
      if (S > 1 && split > 0) {  // previous split's partial must be in C first (bounded wait)
        bool ready = true;
        if (lane == 0) {
          const uint64_t t0 = globaltimer();
          while (ld_acquire_gpu_s32(p.splitk_flags + tile) < 16 * split) {
            if (globaltimer() - t0 > TT_WAIT_TIMEOUT_NS || *reinterpret_cast<volatile int*>(p.status) != 0) {
              atomicCAS(p.status, 0, static_cast<int>(kTimeoutOther));
              ready = false;
              break;
            }
            __nanosleep(128);
          }
        }
        ok = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
        __threadfence();
      }
      const int row_local = mb * 256 + static_cast<int>(crank) * 128 + q * 32 + lane;
      const int row = (GROUP == GROUP_K) ? grp * p.c_grp_rows + row_local : row_local;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN2);
      if (ok)
        epilogue_row<BN2, EPI>(p, t_row, nb, row, row_local < M, alpha, col_half * (OUT_BN_T / 2),
                               (col_half + 1) * (OUT_BN_T / 2));
      if (S > 1) {  // count this warp's rows as added
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.splitk_flags + tile, 1);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&acc_empty[acc]);
        else mbar_arrive_remote(acc_empty0_leader + static_cast<uint32_t>(acc) * 8u);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();  // every MMA retired and every TMEM read done, in both CTAs
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

// ---------------------------------------------------------------------------- host

template <int BN, int STAGES>
constexpr size_t smem_bytes() {
  return static_cast<size_t>(STAGES) * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, int GROUP = GROUP_NONE>
void launch_cfg(const Params& p, const CUtensorMap& ta, const CUtensorMap& tb, int device, cudaStream_t st) {
  constexpr size_t smem = smem_bytes<BN, STAGES>();
  auto kern = gemm_kernel<BN, STAGES, A_MN, B_MN, EPI, GROUP>;
  TT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  constexpr int OUT_BN = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  // GROUP_M: p.M is the row capacity (an upper bound of the device-side total).
  const long num_m = (p.M + BM - 1) / BM;
  const long num_tiles = (GROUP == GROUP_SYM) ? num_m * (num_m + 1) / 2 * p.n_groups
                                              : num_m * ((p.N + OUT_BN - 1) / OUT_BN) *
                                                    ((GROUP == GROUP_K || GROUP == GROUP_BATCH) ? p.n_groups : 1);
  const int grid = static_cast<int>(std::max(1L, std::min(num_tiles, static_cast<long>(num_sms(device)))));
  kern<<<grid, NUM_THREADS, smem, st>>>(ta, tb, p);
  TT_CUDA_CHECK(cudaGetLastError());
}

template <bool A_MN, bool B_MN, int EPI, int GROUP = GROUP_NONE>
void launch_bn(int bn, const Params& p, const CUtensorMap& ta, const CUtensorMap& tb, int device, cudaStream_t st) {
  if constexpr (EPI == EPI_SWIGLU) {
    launch_cfg<256, 4, A_MN, B_MN, EPI, GROUP>(p, ta, tb, device, st);
  } else {
    if (bn == 256)
      launch_cfg<256, 4, A_MN, B_MN, EPI, GROUP>(p, ta, tb, device, st);
    else
      launch_cfg<128, 6, A_MN, B_MN, EPI, GROUP>(p, ta, tb, device, st);
  }
}

template <bool A_MN, bool B_MN, int EPI, int GROUP = GROUP_NONE>
void launch_pair(const Params& p, const CUtensorMap& ta, const CUtensorMap& tb, int device, cudaStream_t st) {
  constexpr size_t smem = static_cast<size_t>(STAGES2) * (PAIR_A_BYTES + PAIR_B_BYTES) + 1024 + 256;
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI, GROUP>;
  TT_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  constexpr int OUT_BN = (EPI == EPI_SWIGLU) ? BN2 / 2 : BN2;
  const long tiles = static_cast<long>((p.M + 255) / 256) * ((p.N + OUT_BN - 1) / OUT_BN) *
                     ((GROUP != GROUP_K && EPI == EPI_F32_ACC && p.split_k > 1) ? p.split_k : 1) *
                     (GROUP == GROUP_K ? p.n_groups : 1);
  const long pairs = std::max(1L, std::min(tiles, static_cast<long>(num_sms(device) / 2)));
  kern<<<static_cast<unsigned>(2 * pairs), PAIR_THREADS, smem, st>>>(ta, tb, p);
  TT_CUDA_CHECK(cudaGetLastError());
}

template <int EPI>
static void dispatch_pair(bool a_mn, bool b_mn, const Params& p, const CUtensorMap& ta, const CUtensorMap& tb,
                          int device, cudaStream_t st) {
  if (!a_mn && !b_mn)
    launch_pair<false, false, EPI>(p, ta, tb, device, st);
  else if (!a_mn && b_mn)
    launch_pair<false, true, EPI>(p, ta, tb, device, st);
  else if (a_mn && b_mn)
    launch_pair<true, true, EPI>(p, ta, tb, device, st);
  else
    launch_pair<true, false, EPI>(p, ta, tb, device, st);
}

// CTA-pair kernel mode: 0 = never, 1 = when estimated faster (default), 2 = always (M >= 256).
// Initialised from TT_GEMM_PAIR; gemm_set_pair_mode changes it at run time (tests).
static std::atomic<int> g_pair_mode{-1};
static int pair_mode() {
  int v = g_pair_mode.load();
  if (v < 0) {
    const char* e = std::getenv("TT_GEMM_PAIR");
    v = (e == nullptr || e[0] == '\0') ? 1 : std::atoi(e);
    g_pair_mode.store(v);
  }
  return v;
}

// Split count for the fp32-accumulate pair kernel.  Each extra split re-reads and rewrites
// the whole fp32 output and serialises one more epilogue per tile, so split only when the
// 256x256 tiles leave most of the last wave idle (utilisation < 0.8), and take the
// smallest split count that reaches 0.85 with >= 32 k-blocks per split.
static int choose_split_k(int M, int N, int K, int device) {
  if (pair_mode() == 0 || M < 256) return 1;
  const long slots = num_sms(device) / 2;
  const long tiles = static_cast<long>((M + 255) / 256) * ((N + BN2 - 1) / BN2);
  auto util = [&](int s) {
    const long u = tiles * s;
    return static_cast<double>(u) / static_cast<double>(((u + slots - 1) / slots) * slots);
  };
  if (util(1) >= 0.8) return 1;
  const int num_k = (K + BK - 1) / BK;
  for (int s = 2; s <= 4; ++s) {
    if (num_k / s < 32) break;
    if (util(s) >= 0.85) return s;
  }
  return 1;
}

// Estimated efficiency of the pair kernel (256 x 256 tiles on SMs/2 clusters) vs the best
// single-CTA tile (which also pays ~15 % more operand traffic per flop).
static bool use_pair(int M, int N, int out_bn_pair, int device) {
  const int mode = pair_mode();
  if (mode == 0 || M < 256) return false;
  if (mode >= 2) return true;
  const int sms = num_sms(device);
  auto util = [](long tiles, long slots) {
    const long waves = (tiles + slots - 1) / slots;
    return static_cast<double>(tiles) / static_cast<double>(waves * slots);
  };
  const long t2 = static_cast<long>((M + 255) / 256) * ((N + out_bn_pair - 1) / out_bn_pair);
  const double e2 = util(t2, sms / 2) * static_cast<double>(N) / (((N + out_bn_pair - 1) / out_bn_pair) * out_bn_pair);
  double e1 = 0.0;
  for (int bn : {128, 256}) {
    const long t1 = static_cast<long>((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    const double e = util(t1, sms) * static_cast<double>(N) / (((N + bn - 1) / bn) * bn) * (bn == 256 ? 0.85 : 0.78);
    e1 = std::max(e1, e);
  }
  return e2 >= e1;
}

// Pick the N tile: prefer 256 unless 128 gives clearly fewer idle SM-slots.
static int choose_bn(int M, int N, int device) {
  const int sms = num_sms(device);
  auto eff = [&](int bn) {
    const long tiles = static_cast<long>((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    const long waves = (tiles + sms - 1) / sms;
    const double util = static_cast<double>(tiles) / static_cast<double>(waves * sms);
    const double colwaste = static_cast<double>(N) / static_cast<double>(((N + bn - 1) / bn) * bn);
    return util * colwaste * (bn == 256 ? 1.0 : 0.93);  // 128-wide tiles re-read A twice as often
  };
  return eff(256) >= eff(128) ? 256 : 128;
}

static CUtensorMap operand_map(const torch::Tensor& t, bool mn_major, int rows_box) {
  // K-major operand: tensor [rows, K] (row stride t.stride(0)); box {BK, rows_box}.
  // MN-major operand: tensor [K, rows] ; box {64, BK}.
  const uint64_t inner = static_cast<uint64_t>(t.size(1));
  const uint64_t outer = static_cast<uint64_t>(t.size(0));
  const uint64_t stride = static_cast<uint64_t>(t.stride(0)) * 2;
  TT_CHECK(t.stride(1) == 1, "GEMM operands must have unit inner stride");
  if (!mn_major) return make_tmap_2d_bf16(t.data_ptr(), inner, outer, stride, BK, rows_box);
  return make_tmap_2d_bf16(t.data_ptr(), inner, outer, stride, 64, BK);
}

template <int EPI>
static void dispatch(bool a_mn, bool b_mn, int bn, const Params& p, const CUtensorMap& ta, const CUtensorMap& tb,
                     int device, cudaStream_t st) {
  if (!a_mn && !b_mn)
    launch_bn<false, false, EPI>(bn, p, ta, tb, device, st);
  else if (!a_mn && b_mn)
    launch_bn<false, true, EPI>(bn, p, ta, tb, device, st);
  else if (a_mn && b_mn)
    launch_bn<true, true, EPI>(bn, p, ta, tb, device, st);
  else
    launch_bn<true, false, EPI>(bn, p, ta, tb, device, st);
}

static Params base_params(int M, int N, int K, const torch::Tensor& out, double alpha,
                          const c10::optional<torch::Tensor>& alpha_t, int device) {
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = out.data_ptr();
  p.ldc = static_cast<int>(out.stride(0));
  p.alpha = static_cast<float>(alpha);
  p.alpha_ptr = nullptr;
  if (alpha_t.has_value()) {
    TT_CHECK(alpha_t->is_cuda() && alpha_t->scalar_type() == torch::kFloat32 && alpha_t->numel() == 1,
             "alpha tensor must be a 1-element float32 CUDA tensor");
    p.alpha_ptr = alpha_t->data_ptr<float>();
  }
  p.status = device_status_ptr(device);
  return p;
}

}  // namespace gemm

// C (+)= alpha * op(A) op(B)^T.
//   a: [M, K] (K-major) or [K, M] (a_mn);  b: [N, K] (K-major) or [K, N] (b_mn)
//   c: [M, N] bf16 (overwritten) or fp32 (overwritten, or accumulated if `accumulate`).
void gemm_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool a_mn, bool b_mn, bool accumulate, double alpha,
             c10::optional<torch::Tensor> alpha_t, int64_t bn) {
  using namespace gemm;
  check_cuda_bf16(a, "a");
  check_cuda_bf16(b, "b");
  TT_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm expects 2-D tensors");
  const int M = static_cast<int>(a_mn ? a.size(1) : a.size(0));
  const int K = static_cast<int>(a_mn ? a.size(0) : a.size(1));
  const int N = static_cast<int>(b_mn ? b.size(1) : b.size(0));
  const int Kb = static_cast<int>(b_mn ? b.size(0) : b.size(1));
  TT_CHECK(K == Kb, "gemm: reduction dims differ");
  TT_CHECK(c.size(0) == M && c.size(1) == N && c.stride(1) == 1, "gemm: bad output shape/stride");
  TT_CHECK(c.is_cuda() && c.device() == a.device() && b.device() == a.device(), "gemm: device mismatch");
  const bool out_bf16 = c.scalar_type() == torch::kBFloat16;
  TT_CHECK(out_bf16 || c.scalar_type() == torch::kFloat32, "gemm: output must be bf16 or fp32");
  TT_CHECK(!(accumulate && out_bf16), "gemm: accumulate needs an fp32 output");
  TT_CHECK(c.stride(0) % (out_bf16 ? 8 : 4) == 0 && reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0,
           "gemm: output rows must be 16-byte aligned");
  if (M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int device = a.get_device();
  if (K == 0) {
    if (!accumulate) c.zero_();
    return;
  }
  cudaStream_t st = cur_stream();
  // Deterministic split-K (fp32 accumulate only): when the pair tiles fill few waves and
  // the reduction is long, e.g. the q|k|v weight gradient (96 tiles, K = 16384).
  const int splits = (accumulate && bn != 128 && bn != 256) ? choose_split_k(M, N, K, device) : 1;
  if (bn == 1 || splits > 1 || (bn == 0 && use_pair(M, N, BN2, device))) {  // bn == 1: the CTA-pair kernel
    const CUtensorMap ta = operand_map(a, a_mn, BM);
    const CUtensorMap tb = operand_map(b, b_mn, 128);
    Params p = base_params(M, N, K, c, alpha, alpha_t, device);
    torch::Tensor flags;
    if (splits > 1) {
      const int64_t tiles = static_cast<int64_t>((M + 255) / 256) * ((N + BN2 - 1) / BN2);
      flags = torch::zeros({tiles}, torch::TensorOptions().dtype(torch::kInt32).device(a.device()));
      p.split_k = splits;
      p.splitk_flags = flags.data_ptr<int>();
    }
    if (out_bf16)
      dispatch_pair<EPI_BF16>(a_mn, b_mn, p, ta, tb, device, st);
    else if (accumulate)
      dispatch_pair<EPI_F32_ACC>(a_mn, b_mn, p, ta, tb, device, st);
    else
      dispatch_pair<EPI_F32>(a_mn, b_mn, p, ta, tb, device, st);
    return;
  }
  const int use_bn = (bn == 128 || bn == 256) ? static_cast<int>(bn) : choose_bn(M, N, device);
  const CUtensorMap ta = operand_map(a, a_mn, BM);
  const CUtensorMap tb = operand_map(b, b_mn, use_bn);
  Params p = base_params(M, N, K, c, alpha, alpha_t, device);
  if (out_bf16)
    dispatch<EPI_BF16>(a_mn, b_mn, use_bn, p, ta, tb, device, st);
  else if (accumulate)
    dispatch<EPI_F32_ACC>(a_mn, b_mn, use_bn, p, ta, tb, device, st);
  else
    dispatch<EPI_F32>(a_mn, b_mn, use_bn, p, ta, tb, device, st);
}

// Newton-Schulz building block (Muon): C = alpha * A op(B)^T + beta * addend, bf16 out,
// for `batch` independent products of one shape stacked along the rows:
//   a: [batch * M, K] K-major;  b: [batch * N, K] (K-major) or [batch * K, N] (b_mn);
//   c and addend (optional): bf16 [batch * M, N].
//   symmetric: each product is known to be symmetric (B == A giving A A^T, or A symmetric
//   giving A A = A A^T): only the 128x128 tiles on or above the diagonal are computed and
//   each is mirrored, which halves the work of X X^T and of A^2.  The addend must then be
//   symmetric as well (it is A itself in b*A + c*A^2).
void gemm_axpby_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool b_mn, double alpha,
                   c10::optional<torch::Tensor> addend, double beta, bool symmetric, int64_t batch) {
  using namespace gemm;
  check_cuda_bf16(a, "a");
  check_cuda_bf16(b, "b");
  check_cuda_bf16(c, "c");
  TT_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm_axpby expects 2-D tensors");
  TT_CHECK(batch >= 1 && a.size(0) % batch == 0 && b.size(0) % batch == 0 && c.size(0) % batch == 0,
           "gemm_axpby: row counts must be divisible by the batch");
  const int M = static_cast<int>(a.size(0) / batch), K = static_cast<int>(a.size(1));
  const int N = static_cast<int>(b_mn ? b.size(1) : b.size(0) / batch);
  TT_CHECK(K == static_cast<int>(b_mn ? b.size(0) / batch : b.size(1)), "gemm_axpby: reduction dims differ");
  TT_CHECK(c.size(0) == batch * M && c.size(1) == N && c.stride(1) == 1 && c.stride(0) % 8 == 0 &&
               reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0,
           "gemm_axpby: output must be [batch * M, N] with 16-byte aligned rows");
  TT_CHECK(!symmetric || (M == N && !b_mn), "gemm_axpby: a symmetric product needs M == N and K-major B");
  if (M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int device = a.get_device();
  Params p = base_params(M, N, K, c, alpha, c10::nullopt, device);
  p.beta = static_cast<float>(beta);
  p.n_groups = static_cast<int>(batch);
  p.a_grp_rows = M;
  p.b_grp_rows = b_mn ? K : N;
  p.c_grp_rows = M;
  if (addend.has_value()) {
    check_cuda_bf16(*addend, "addend");
    TT_CHECK(addend->dim() == 2 && addend->size(0) == batch * M && addend->size(1) == N && addend->stride(1) == 1 &&
                 addend->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(addend->data_ptr()) % 16 == 0,
             "gemm_axpby: addend must be bf16 [batch * M, N] with 16-byte aligned rows");
    p.aux = reinterpret_cast<const __nv_bfloat16*>(addend->data_ptr());
    p.ld_aux = static_cast<int>(addend->stride(0));
  }
  cudaStream_t st = cur_stream();
  const CUtensorMap ta = operand_map(a, false, BM);
  if (symmetric) {
    const CUtensorMap tb = operand_map(b, false, 128);
    if (addend.has_value())
      launch_cfg<128, 6, false, false, EPI_AXPBY, GROUP_SYM>(p, ta, tb, device, st);
    else
      launch_cfg<128, 6, false, false, EPI_BF16, GROUP_SYM>(p, ta, tb, device, st);
    return;
  }
  TT_CHECK(addend.has_value(), "gemm_axpby: a plain product goes through gemm()");
  if (batch == 1 && use_pair(M, N, BN2, device)) {
    const CUtensorMap tb = operand_map(b, b_mn, 128);
    if (b_mn) launch_pair<false, true, EPI_AXPBY>(p, ta, tb, device, st);
    else launch_pair<false, false, EPI_AXPBY>(p, ta, tb, device, st);
    return;
  }
  const int bn = choose_bn(M, N, device);
  const CUtensorMap tb = operand_map(b, b_mn, bn);
  if (b_mn) launch_bn<false, true, EPI_AXPBY, GROUP_BATCH>(bn, p, ta, tb, device, st);
  else launch_bn<false, false, EPI_AXPBY, GROUP_BATCH>(bn, p, ta, tb, device, st);
}

void gemm_set_pair_mode(int64_t mode) { gemm::g_pair_mode.store(static_cast<int>(mode)); }
int64_t gemm_pair_mode() { return gemm::pair_mode(); }

// out[M, I] = silu(x Wg^T) * (x Wu^T) with w_gu = [Wg; Wu] ([2I, K], K-major).
// If gu_out is given, also stores the pre-activations g|u ([M, 2I]) for backward.
void gemm_swiglu_op(torch::Tensor x, torch::Tensor w_gu, torch::Tensor out, c10::optional<torch::Tensor> gu_out) {
  using namespace gemm;
  check_cuda_bf16(x, "x");
  check_cuda_bf16(w_gu, "w_gu");
  check_cuda_bf16(out, "out");
  const int M = static_cast<int>(x.size(0));
  const int K = static_cast<int>(x.size(1));
  TT_CHECK(w_gu.size(1) == K && w_gu.size(0) % 2 == 0, "swiglu: weight must be [2I, K]");
  const int I = static_cast<int>(w_gu.size(0) / 2);
  TT_CHECK(out.size(0) == M && out.size(1) == I && out.stride(1) == 1 && out.stride(0) % 8 == 0,
           "swiglu: bad output");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  const int device = x.get_device();
  const CUtensorMap ta = operand_map(x, false, BM);
  const CUtensorMap tb = make_tmap_2d_bf16(w_gu.data_ptr(), static_cast<uint64_t>(K), static_cast<uint64_t>(2 * I),
                                           static_cast<uint64_t>(w_gu.stride(0)) * 2, BK, 128);
  Params p = base_params(M, I, K, out, 1.0, c10::nullopt, device);
  p.b_row_offset2 = I;
  if (gu_out.has_value()) {
    check_cuda_bf16(*gu_out, "gu_out");
    TT_CHECK(gu_out->size(0) == M && gu_out->size(1) == 2 * I && gu_out->stride(0) % 8 == 0, "swiglu: bad gu_out");
    p.aux_out = reinterpret_cast<__nv_bfloat16*>(gu_out->data_ptr());
    p.ld_aux_out = static_cast<int>(gu_out->stride(0));
  }
  TT_CHECK(I % 8 == 0, "swiglu: intermediate size must be a multiple of 8");
  if (use_pair(M, I, BN2 / 2, device)) {
    launch_pair<false, false, EPI_SWIGLU>(p, ta, tb, device, cur_stream());
    return;
  }
  launch_bn<false, false, EPI_SWIGLU>(256, p, ta, tb, device, cur_stream());
}

// d(g|u)[M, 2I] from dy[M, D], w_down[D, I] and the saved pre-activations gu[M, 2I]:
//   dact = dy @ w_down ; dg = dact * u * silu'(g) ; du = dact * silu(g)
void gemm_dswiglu_op(torch::Tensor dy, torch::Tensor w_down, torch::Tensor gu, torch::Tensor dgu, double alpha) {
  using namespace gemm;
  check_cuda_bf16(dy, "dy");
  check_cuda_bf16(w_down, "w_down");
  check_cuda_bf16(gu, "gu");
  check_cuda_bf16(dgu, "dgu");
  const int M = static_cast<int>(dy.size(0));
  const int D = static_cast<int>(dy.size(1));
  TT_CHECK(w_down.size(0) == D, "dswiglu: w_down must be [D, I]");
  const int I = static_cast<int>(w_down.size(1));
  TT_CHECK(gu.size(0) == M && gu.size(1) == 2 * I && dgu.size(0) == M && dgu.size(1) == 2 * I, "dswiglu: bad shapes");
  TT_CHECK(I % 64 == 0, "dswiglu: intermediate size must be a multiple of 64");
  TT_CHECK(gu.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(gu.data_ptr()) % 16 == 0 && gu.stride(1) == 1,
           "dswiglu: gu rows must be 16-byte aligned");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(dy.device());
  const int device = dy.get_device();
  const bool pair = use_pair(M, I, BN2, device);
  const int bn = pair ? 128 : choose_bn(M, I, device);
  const CUtensorMap ta = operand_map(dy, false, BM);
  const CUtensorMap tb = operand_map(w_down, true, bn);
  Params p = base_params(M, I, D, dgu, alpha, c10::nullopt, device);
  p.C = nullptr;
  p.aux = reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr());
  p.ld_aux = static_cast<int>(gu.stride(0));
  p.aux_out = reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr());
  p.ld_aux_out = static_cast<int>(dgu.stride(0));
  if (pair) {
    launch_pair<false, true, EPI_DSWIGLU>(p, ta, tb, device, cur_stream());
    return;
  }
  launch_bn<false, true, EPI_DSWIGLU>(bn, p, ta, tb, device, cur_stream());
}

// ---------------------------------------------------------------------------- grouped (MoE) GEMMs
namespace gemm {
static void check_grp(const torch::Tensor& grp_off, int64_t n_groups, const torch::Tensor& like) {
  TT_CHECK(grp_off.is_cuda() && grp_off.scalar_type() == torch::kInt32 && grp_off.numel() == n_groups + 1,
           "grouped gemm: grp_off must be int32 CUDA [n_groups + 1]");
  TT_CHECK(grp_off.device() == like.device(), "grouped gemm: grp_off on another device");
  TT_CHECK(n_groups >= 1, "grouped gemm: n_groups >= 1");
}
}  // namespace gemm

// C_rows[cap, N] (bf16) = A_rows[cap, K] . B_e^T for the expert e owning each 128-row tile.
//   b K-major: [n_groups * b_grp_rows, K], expert e's rows start at e * b_grp_rows.
//   b MN-major: [rows, N] indexed by k; k-blocks < b_split_k/64 at e*b_grp_rows + k, the rest at
//   b_off2 + e*b_grp_rows + (k - b_split_k) (gate|up weights stored as two stacked tensors).
// pair: the caller laid the segments out on 256-row boundaries, so the CTA-pair kernel
// may run the GEMM (TT_GEMM_PAIR=0 still forces the single-CTA kernel).
void moe_gemm_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_off, int64_t n_groups,
                 bool b_mn, int64_t b_grp_rows, int64_t b_split_k, int64_t b_off2, bool pair,
                 c10::optional<torch::Tensor> row_ptr) {
  using namespace gemm;
  check_cuda_bf16(a, "a");
  check_cuda_bf16(b, "b");
  check_cuda_bf16(c, "c");
  check_grp(grp_off, n_groups, a);
  const int M = static_cast<int>(a.size(0));
  const int K = static_cast<int>(a.size(1));
  const int N = static_cast<int>(c.size(1));
  TT_CHECK(c.size(0) == M && c.stride(1) == 1 && c.stride(0) % 8 == 0, "moe_gemm: bad output");
  if (row_ptr.has_value()) {
    TT_CHECK(row_ptr->is_cuda() && row_ptr->scalar_type() == torch::kInt64 && row_ptr->numel() >= M &&
                 row_ptr->is_contiguous(),
             "moe_gemm: row_ptr must be a contiguous CUDA int64 tensor with one address per output row");
  }
  TT_CHECK(b_mn ? b.size(1) == N : b.size(1) == K, "moe_gemm: B shape");
  TT_CHECK(b_split_k % BK == 0 && b_grp_rows % (b_mn ? BK : 1) == 0, "moe_gemm: group offsets must be 64-aligned");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int device = a.get_device();
  const bool use2 = pair && pair_mode() != 0 && M >= 256;
  const int bn = use2 ? 128 : choose_bn(M, N, device);
  const CUtensorMap ta = operand_map(a, false, BM);
  const CUtensorMap tb = operand_map(b, b_mn, bn);
  Params p = base_params(M, N, K, c, 1.0, c10::nullopt, device);
  p.grp_off = grp_off.data_ptr<int>();
  p.n_groups = static_cast<int>(n_groups);
  p.b_grp_rows = static_cast<int>(b_grp_rows);
  p.b_split_kb = b_split_k > 0 ? static_cast<int>(b_split_k / BK) : (1 << 30);
  p.b_off2 = static_cast<int>(b_off2);
  p.row_ptr = row_ptr.has_value() ? reinterpret_cast<const long long*>(row_ptr->data_ptr<int64_t>()) : nullptr;
  if (use2) {
    if (b_mn) launch_pair<false, true, EPI_BF16, GROUP_M>(p, ta, tb, device, cur_stream());
    else launch_pair<false, false, EPI_BF16, GROUP_M>(p, ta, tb, device, cur_stream());
    return;
  }
  if (b_mn)
    launch_bn<false, true, EPI_BF16, GROUP_M>(bn, p, ta, tb, device, cur_stream());
  else
    launch_bn<false, false, EPI_BF16, GROUP_M>(bn, p, ta, tb, device, cur_stream());
}

// act[cap, I] = silu(x_e Wg_e^T) * (x_e Wu_e^T) per expert; w_gu = [Wg (n_groups*I rows); Wu (same)].
void moe_gemm_swiglu_op(torch::Tensor x, torch::Tensor w_gu, torch::Tensor out, torch::Tensor gu_out,
                        torch::Tensor grp_off, int64_t n_groups, bool pair) {
  using namespace gemm;
  check_cuda_bf16(x, "x");
  check_cuda_bf16(w_gu, "w_gu");
  check_cuda_bf16(out, "out");
  check_cuda_bf16(gu_out, "gu_out");
  check_grp(grp_off, n_groups, x);
  const int M = static_cast<int>(x.size(0));
  const int K = static_cast<int>(x.size(1));
  const int I = static_cast<int>(out.size(1));
  TT_CHECK(w_gu.size(0) == 2 * n_groups * I && w_gu.size(1) == K, "moe_swiglu: w_gu must be [2*E*I, K]");
  TT_CHECK(out.size(0) == M && out.stride(0) % 8 == 0 && gu_out.size(0) == M && gu_out.size(1) == 2 * I &&
               gu_out.stride(0) % 8 == 0 && I % 8 == 0, "moe_swiglu: bad outputs");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  const int device = x.get_device();
  const CUtensorMap ta = operand_map(x, false, BM);
  const CUtensorMap tb = make_tmap_2d_bf16(w_gu.data_ptr(), static_cast<uint64_t>(K), static_cast<uint64_t>(w_gu.size(0)),
                                           static_cast<uint64_t>(w_gu.stride(0)) * 2, BK, 128);
  Params p = base_params(M, I, K, out, 1.0, c10::nullopt, device);
  p.b_row_offset2 = static_cast<int>(n_groups * I);
  p.aux_out = reinterpret_cast<__nv_bfloat16*>(gu_out.data_ptr());
  p.ld_aux_out = static_cast<int>(gu_out.stride(0));
  p.grp_off = grp_off.data_ptr<int>();
  p.n_groups = static_cast<int>(n_groups);
  p.b_grp_rows = I;
  if (pair && pair_mode() != 0 && M >= 256) {
    launch_pair<false, false, EPI_SWIGLU, GROUP_M>(p, ta, tb, device, cur_stream());
    return;
  }
  launch_bn<false, false, EPI_SWIGLU, GROUP_M>(256, p, ta, tb, device, cur_stream());
}

// d(g|u)[cap, 2I] from dy_rows[cap, D], w_down [n_groups*D, I] and the saved g|u.
void moe_gemm_dswiglu_op(torch::Tensor dy, torch::Tensor w_down, torch::Tensor gu, torch::Tensor dgu,
                         torch::Tensor grp_off, int64_t n_groups, bool pair) {
  using namespace gemm;
  check_cuda_bf16(dy, "dy");
  check_cuda_bf16(w_down, "w_down");
  check_cuda_bf16(gu, "gu");
  check_cuda_bf16(dgu, "dgu");
  check_grp(grp_off, n_groups, dy);
  const int M = static_cast<int>(dy.size(0));
  const int D = static_cast<int>(dy.size(1));
  const int I = static_cast<int>(w_down.size(1));
  TT_CHECK(w_down.size(0) == n_groups * D && D % BK == 0, "moe_dswiglu: w_down must be [E*D, I], D % 64 == 0");
  TT_CHECK(gu.size(0) == M && gu.size(1) == 2 * I && dgu.size(0) == M && dgu.size(1) == 2 * I && I % 64 == 0,
           "moe_dswiglu: bad shapes");
  TT_CHECK(gu.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(gu.data_ptr()) % 16 == 0 && gu.stride(1) == 1,
           "moe_dswiglu: gu rows must be 16-byte aligned");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(dy.device());
  const int device = dy.get_device();
  const bool use2 = pair && pair_mode() != 0 && M >= 256;
  const int bn = use2 ? 128 : choose_bn(M, I, device);
  const CUtensorMap ta = operand_map(dy, false, BM);
  const CUtensorMap tb = operand_map(w_down, true, bn);
  Params p = base_params(M, I, D, dgu, 1.0, c10::nullopt, device);
  p.C = nullptr;
  p.aux = reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr());
  p.ld_aux = static_cast<int>(gu.stride(0));
  p.aux_out = reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr());
  p.ld_aux_out = static_cast<int>(dgu.stride(0));
  p.grp_off = grp_off.data_ptr<int>();
  p.n_groups = static_cast<int>(n_groups);
  p.b_grp_rows = D;
  p.b_split_kb = 1 << 30;
  if (use2) {
    launch_pair<false, true, EPI_DSWIGLU, GROUP_M>(p, ta, tb, device, cur_stream());
    return;
  }
  launch_bn<false, true, EPI_DSWIGLU, GROUP_M>(bn, p, ta, tb, device, cur_stream());
}

// Per-expert weight gradient: C[e*M:(e+1)*M, N] (+)= A_e^T B_e with A [cap, M], B [cap, N]
// (token rows; the reduction covers expert e's segment only).  C is fp32.
// pair: CTA-pair kernel (256 x 256 tiles per expert); any segment alignment of 64 rows works,
// since the reduction runs over whole k-blocks of each expert's token segment.
void moe_gemm_wgrad_op(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_off, int64_t n_groups,
                       bool accumulate, bool pair) {
  using namespace gemm;
  check_cuda_bf16(a, "a");
  check_cuda_bf16(b, "b");
  check_grp(grp_off, n_groups, a);
  const int M = static_cast<int>(a.size(1));
  const int N = static_cast<int>(b.size(1));
  const int K = static_cast<int>(a.size(0));
  TT_CHECK(b.size(0) == K, "moe_wgrad: token rows differ");
  TT_CHECK(c.scalar_type() == torch::kFloat32 && c.size(0) == n_groups * M && c.size(1) == N && c.stride(1) == 1 &&
               c.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0,
           "moe_wgrad: C must be fp32 [E*M, N] with 16-byte aligned rows");
  const c10::cuda::CUDAGuard guard(a.device());
  const int device = a.get_device();
  if (!accumulate) c.zero_();  // empty experts' tiles are skipped
  if (K == 0) return;
  const bool use2 = pair && pair_mode() != 0;
  const int bn = use2 ? 128 : choose_bn(M, N, device);
  const CUtensorMap ta = operand_map(a, true, BM);
  const CUtensorMap tb = operand_map(b, true, bn);
  Params p = base_params(M, N, K, c, 1.0, c10::nullopt, device);
  p.grp_off = grp_off.data_ptr<int>();
  p.n_groups = static_cast<int>(n_groups);
  p.c_grp_rows = M;
  if (use2) {
    launch_pair<true, true, EPI_F32_ACC, GROUP_K>(p, ta, tb, device, cur_stream());
    return;
  }
  launch_bn<true, true, EPI_F32_ACC, GROUP_K>(bn, p, ta, tb, device, cur_stream());
}

}  // namespace tt
