// Weight-streaming GEMM for a few token rows (decode) on the 5th-gen tensor cores.
//
//   Y[t, n] = sum_k X[t, k] W[n, k]        t < 32 tokens (per group), W large
//
// At decode a GEMM has at most a few dozen token rows, so its cost is streaming W once
// from HBM.  The regular tile kernel puts tokens on the 128-row MMA side (97 % padding)
// and spreads the work as one CTA per 128 or 256 output columns, which leaves SMs idle
// when the weight matrix has few column blocks (an expert-parallel rank's 8 experts, a
// 2048-wide projection).  Here the operands are swapped and the reduction is split:
//
//   * the weight rows are the MMA's M side (128 rows per tile, TMA box 64 x 128) and the
//     tokens its N side (N = 32, TMA box 64 x 32; rows past a group's count are read but
//     never stored), so every byte a CTA loads except the small token tile is weight;
//   * the work unit is (group, half, 128-row block, k-split); the split count is chosen so
//     that there are about three units per SM, and a persistent CTA per SM walks its units
//     with an 8-stage TMA ring (128 KB of weight in flight per SM) and a double-buffered
//     32-column TMEM accumulator, so one unit's epilogue overlaps the next unit's loads;
//   * each unit stores its fp32 partial sums ([split][token row][output column]), and a
//     second small kernel adds the splits in a fixed order (deterministic) and applies the
//     epilogue: bf16 store, SwiGLU (gate and up halves), or the MoE top-k weighted combine.
//
// Grouped mode (MoE experts): token rows are laid out by expert without padding
// (grp_off[g] .. grp_off[g+1], on the device); group g's weights are rows
// half_base[h] + g * group_stride + [0, half_cols) for each half h.  A token routes to an
// expert at most once, so a group never holds more token rows than the batch (<= 32).
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +31 = weight rows).
// Every wait is bounded (status word + early exit), as in the tile GEMM.
#include "common/ptx.cuh"
#include "common/host_utils.h"
#include "runtime/comm_common.cuh"

#include <algorithm>
#include <mutex>

namespace tt {
namespace skinny {

constexpr int BW = 128;  // weight rows per tile (MMA M)
constexpr int BT = 32;   // token columns per tile (MMA N)
constexpr int BK = 64;
constexpr int STAGES = 8;
constexpr int THREADS = 192;
constexpr uint32_t W_BYTES = BW * BK * 2;  // 16 KB
constexpr uint32_t X_BYTES = BT * BK * 2;  // 4 KB
constexpr uint32_t TMEM_COLS = 2 * BT;     // double-buffered accumulator
constexpr uint32_t IDESC = idesc_bf16_f32(BW, BT, false, false);
constexpr size_t SMEM_BYTES = 1024 + STAGES * (W_BYTES + X_BYTES) + 256;

struct Params {
  int K, num_kb;
  int n_groups;
  const int* grp_off;  // [n_groups + 1] token row offsets (device); nullptr: one group of M rows
  int M;
  int halves;          // 1, or 2 when a group's outputs come from two weight ranges (gate | up)
  int half_cols;       // output columns per half
  int half_base0, half_base1;  // first weight row of each half for group 0
  int group_stride;    // weight rows between consecutive groups within a half
  int nrb;             // 128-row blocks per half
  int splits, kb_per_split;
  float* part;         // [splits, rows_cap, ld_part] fp32 partial sums
  int rows_cap, ld_part;
  int* status;
};

// Optional fused publish of a row-parallel all-reduce (SEP inference): the split-sum
// kernel writes its bf16 result straight into this rank's symmetric-heap slot of the
// graph-safe all-reduce (slot = device epoch parity) and its last block signals the peers,
// so only the reducing kernel remains (it waits for every peer's epoch and sums the slots).
struct Publish {
  comm::PeerTable t;
  size_t slot_off;
  long long slot_bytes;
  int on;
};

// Destination of the split-sum kernel's bf16 output: `out` (row stride ld_out), or with a
// publish the heap slot of the coming epoch (contiguous rows of N).
__device__ __forceinline__ __nv_bfloat16* publish_dst(const Publish& pub, __nv_bfloat16* out, int& ld_out, int N,
                                                      uint64_t& e) {
  if (!pub.on) return out;
  e = comm::dev_epoch_next(pub.t);
  ld_out = N;
  return reinterpret_cast<__nv_bfloat16*>(pub.t.base[pub.t.rank] + pub.slot_off +
                                          static_cast<size_t>(e & 1ull) * static_cast<size_t>(pub.slot_bytes));
}

struct Unit {
  int g, h, rb, s;
};

__device__ __forceinline__ Unit unit_of(int u, const Params& p) {
  Unit r;
  r.s = u % p.splits;
  u /= p.splits;
  r.rb = u % p.nrb;
  u /= p.nrb;
  r.h = u % p.halves;
  r.g = u / p.halves;
  return r;
}

__device__ __forceinline__ void group_rows(const Params& p, int g, int& row0, int& cnt) {
  if (p.grp_off == nullptr) {
    row0 = 0;
    cnt = p.M;
  } else {
    row0 = __ldg(p.grp_off + g);
    cnt = __ldg(p.grp_off + g + 1) - row0;
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_ptr(smem_raw, 1024);
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * W_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + STAGES * X_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_units = p.n_groups * p.halves * p.nrb * p.splits;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
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
      uint32_t phase = 0, pending = 0, pending_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x) {
        const Unit t = unit_of(u, p);
        int row0, cnt;
        group_rows(p, t.g, row0, cnt);
        if (cnt <= 0) continue;
        if (cnt > BT) {  // more token rows than one tile holds: the group is skipped
          if (t.h == 0 && t.rb == 0 && t.s == 0) atomicCAS(p.status, 0, static_cast<int>(kBadIndex));
          continue;
        }
        const int kb0 = t.s * p.kb_per_split, kb1 = min(kb0 + p.kb_per_split, p.num_kb);
        const int wrow = (t.h ? p.half_base1 : p.half_base0) + t.g * p.group_stride + t.rb * BW;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], W_BYTES + X_BYTES);
          tma_load_2d(sW + stage * W_BYTES, &tmW, &full[stage], kb * BK, wrow);
          tma_load_2d(sX + stage * X_BYTES, &tmX, &full[stage], kb * BK, row0);
          pending |= (1u << stage);
          pending_phase = (pending_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (pending & (1u << s)) mbar_wait(&full[s], (pending_phase >> s) & 1u, p.status, kTimeoutOther);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x) {
        const Unit t = unit_of(u, p);
        int row0, cnt;
        group_rows(p, t.g, row0, cnt);
        if (cnt <= 0 || cnt > BT) continue;
        const int kb0 = t.s * p.kb_per_split, kb1 = min(kb0 + p.kb_per_split, p.num_kb);
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, p.status, kTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BT);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w_base = smem_u32(sW + stage * W_BYTES);
          const uint32_t x_base = smem_u32(sX + stage * X_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            umma_f16_ss(d_tmem, sdesc_sw128(w_base + j * 32, 16, 1024), sdesc_sw128(x_base + j * 32, 16, 1024), IDESC,
                        (kb > kb0 || j > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, p.status, kTimeoutOther);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;
    const int wl = q * 32 + lane;  // weight row within the tile = output column
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const Unit t = unit_of(u, p);
      int row0, cnt;
      group_rows(p, t.g, row0, cnt);
      if (cnt <= 0 || cnt > BT) continue;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, p.status, kTimeoutAccFull)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BT), r);
      tmem_ld_wait();
      const int col = t.rb * BW + wl;
      if (col < p.half_cols) {
        float* dst = p.part + (static_cast<size_t>(t.s) * p.rows_cap + row0) * p.ld_part + t.h * p.half_cols + col;
#pragma unroll
        for (int i = 0; i < BT; ++i)
          if (i < cnt) dst[static_cast<size_t>(i) * p.ld_part] = __uint_as_float(r[i]);
      }
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

// ---------------------------------------------------------------------------- split sums
__device__ __forceinline__ float4 sum_splits4(const float* part, int splits, size_t split_stride, size_t off) {
  float4 a = *reinterpret_cast<const float4*>(part + off);
  for (int s = 1; s < splits; ++s) {
    const float4 b = *reinterpret_cast<const float4*>(part + s * split_stride + off);
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
  }
  return a;
}

// out[r, n] = bf16(sum_s part[s, r, n]), r < M, n < N (N % 4 == 0).
__global__ void reduce_bf16_kernel(const float* __restrict__ part, int splits, int rows_cap, int ld, int M, int N,
                                   __nv_bfloat16* __restrict__ out, int ld_out, const Publish pub) {
  uint64_t e = 0;
  out = publish_dst(pub, out, ld_out, N, e);
  const int n4 = N / 4;
  const size_t total = static_cast<size_t>(M) * n4;
  const size_t ss = static_cast<size_t>(rows_cap) * ld;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / n4), c = static_cast<int>(i % n4) * 4;
    const float4 v = sum_splits4(part, splits, ss, static_cast<size_t>(r) * ld + c);
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(r) * ld_out + c) = o;
  }
  if (pub.on) comm::grid_last_block(pub.t, [&]() { comm::signal_peers(pub.t, e); });
}

// act[r, j] = bf16(silu(g) * u) with g, u the split sums of columns j and I + j; rows below
// the device-side row count only.
__global__ void reduce_swiglu_kernel(const float* __restrict__ part, int splits, int rows_cap, int I,
                                     const int* __restrict__ rows_dev, __nv_bfloat16* __restrict__ act, int ld_act) {
  const int rows = *rows_dev;
  const int i4 = I / 4;
  const size_t total = static_cast<size_t>(rows) * i4;
  const int ld = 2 * I;
  const size_t ss = static_cast<size_t>(rows_cap) * ld;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / i4), c = static_cast<int>(i % i4) * 4;
    const float4 g = sum_splits4(part, splits, ss, static_cast<size_t>(r) * ld + c);
    const float4 u = sum_splits4(part, splits, ss, static_cast<size_t>(r) * ld + I + c);
    auto sw = [](float gv, float uv) { return gv / (1.0f + __expf(-gv)) * uv; };
    uint2 o;
    o.x = pack_bf16x2(sw(g.x, u.x), sw(g.y, u.y));
    o.y = pack_bf16x2(sw(g.z, u.z), sw(g.w, u.w));
    *reinterpret_cast<uint2*>(act + static_cast<size_t>(r) * ld_act + c) = o;
  }
}

// out[n, :] = bf16(sum_j w[n, j] * sum_s part[s, slot[n, j], :]) over the token's k pairs;
// pairs whose slot is at or past *row_limit (computed on another rank) are skipped.
// One CTA per token, a thread per 4 columns.
__global__ void reduce_combine_kernel(const float* __restrict__ part, int splits, int rows_cap, int H,
                                      const int* __restrict__ slot, const float* __restrict__ w, int k,
                                      const int* __restrict__ row_limit, __nv_bfloat16* __restrict__ out, int ld_out,
                                      const Publish pub) {
  uint64_t e = 0;
  out = publish_dst(pub, out, ld_out, H, e);
  const int n = blockIdx.x;
  const int limit = row_limit != nullptr ? *row_limit : 0x7fffffff;
  const size_t ss = static_cast<size_t>(rows_cap) * H;
  for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const int r = slot[n * k + j];
      if (r < 0 || r >= limit || r >= rows_cap) continue;
      const float wj = w != nullptr ? w[n * k + j] : 1.0f;
      const float4 v = sum_splits4(part, splits, ss, static_cast<size_t>(r) * H + c);
      acc.x = fmaf(wj, v.x, acc.x);
      acc.y = fmaf(wj, v.y, acc.y);
      acc.z = fmaf(wj, v.z, acc.z);
      acc.w = fmaf(wj, v.w, acc.w);
    }
    uint2 o;
    o.x = pack_bf16x2(acc.x, acc.y);
    o.y = pack_bf16x2(acc.z, acc.w);
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(n) * ld_out + c) = o;
  }
  if (pub.on) comm::grid_last_block(pub.t, [&]() { comm::signal_peers(pub.t, e); });
}

// ---------------------------------------------------------------------------- host side
// About three work units per SM; at least two k-blocks per unit.
static void choose_splits(Params& p, int device) {
  const int units1 = std::max(1, p.n_groups * p.halves * p.nrb);
  const int target = 3 * num_sms(device);
  int s = std::max(1, (target + units1 - 1) / units1);
  s = std::min(s, std::max(1, p.num_kb / 2));
  p.kb_per_split = (p.num_kb + s - 1) / s;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
}

static void launch(const torch::Tensor& w, const torch::Tensor& x, const Params& p, int device) {
  const CUtensorMap tw = make_tmap_2d_bf16(w.data_ptr(), static_cast<uint64_t>(p.K), static_cast<uint64_t>(w.size(0)),
                                           static_cast<uint64_t>(w.stride(0)) * 2, BK, BW);
  const CUtensorMap tx = make_tmap_2d_bf16(x.data_ptr(), static_cast<uint64_t>(p.K), static_cast<uint64_t>(x.size(0)),
                                           static_cast<uint64_t>(x.stride(0)) * 2, BK, BT);
  static std::once_flag once[64];
  std::call_once(once[device & 63], [] {
    TT_CUDA_CHECK(cudaFuncSetAttribute(skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(SMEM_BYTES)));
  });
  const int units = p.n_groups * p.halves * p.nrb * p.splits;
  const int grid = std::max(1, std::min(units, num_sms(device)));
  skinny_kernel<<<grid, THREADS, SMEM_BYTES, cur_stream()>>>(tw, tx, p);
  TT_CUDA_CHECK(cudaGetLastError());
}

static void check_operand(const torch::Tensor& t, const char* name) {
  check_cuda_bf16(t, name);
  TT_CHECK(t.dim() == 2 && t.stride(1) == 1 && t.stride(0) % 8 == 0 &&
               reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
           std::string(name) + ": rows of a 16-byte aligned row-major matrix expected");
}

// Every operand of one call must live on the launching device (the first operand's).
static void check_device(const torch::Tensor& t, int device, const char* name) {
  TT_CHECK(t.is_cuda() && t.get_device() == device, std::string(name) + ": must be on the operands' CUDA device");
}

// Publish target (gid >= 0): a heap slot pair of a graph-safe all-reduce (see Publish);
// `bytes` is the size of the output that will be written there.
static Publish make_publish(int64_t gid, int64_t slot_off, int64_t slot_bytes, int64_t bytes, int device) {
  Publish pub{};
  if (gid < 0) return pub;
  TT_CHECK(comm::group_device(gid) == device, "skinny publish: heap on another device");
  TT_CHECK(slot_off % 16 == 0 && slot_bytes % 16 == 0 && bytes <= slot_bytes &&
               slot_off + 2 * slot_bytes <= static_cast<int64_t>(comm::group_bytes(gid)),
           "skinny publish: slot outside the heap or too small");
  pub.t = comm::group_table(gid);
  pub.slot_off = static_cast<size_t>(slot_off);
  pub.slot_bytes = slot_bytes;
  pub.on = 1;
  return pub;
}

static Params base_params(int K, int device) {
  Params p{};
  p.K = K;
  p.num_kb = (K + BK - 1) / BK;
  p.status = device_status_ptr(device);
  return p;
}

}  // namespace skinny

// y[M, N] = x[M, K] w[N, K]^T for M <= 32 (decode-sized batches).
void skinny_linear_op(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t publish_gid, int64_t slot_off,
                      int64_t slot_bytes) {
  using namespace skinny;
  check_operand(x, "x");
  check_operand(w, "w");
  check_cuda_bf16(out, "out");
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1)), N = static_cast<int>(w.size(0));
  TT_CHECK(M <= BT, "skinny_linear: at most 32 rows");
  TT_CHECK(w.size(1) == K && K % 8 == 0 && N % 4 == 0, "skinny_linear: w [N, K] with K % 8 == 0 and N % 4 == 0");
  TT_CHECK(out.size(0) == M && out.size(1) == N && out.stride(1) == 1 && out.stride(0) % 4 == 0 &&
               reinterpret_cast<uintptr_t>(out.data_ptr()) % 8 == 0,
           "skinny_linear: out [M, N]");
  check_device(w, x.get_device(), "skinny_linear w");
  check_device(out, x.get_device(), "skinny_linear out");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  const int device = x.get_device();
  Params p = base_params(K, device);
  p.n_groups = 1;
  p.grp_off = nullptr;
  p.M = M;
  p.halves = 1;
  p.half_cols = N;
  p.half_base0 = p.half_base1 = 0;
  p.group_stride = 0;
  p.nrb = (N + BW - 1) / BW;
  choose_splits(p, device);
  torch::Tensor part = torch::empty({p.splits, M, N}, x.options().dtype(torch::kFloat32));
  p.part = part.data_ptr<float>();
  p.rows_cap = M;
  p.ld_part = N;
  launch(w, x, p, device);
  const int threads = 256;
  const int blocks = std::max(1, std::min(num_sms(device) * 4, (M * N / 4 + threads - 1) / threads));
  const Publish pub = make_publish(publish_gid, slot_off, slot_bytes, static_cast<int64_t>(M) * N * 2, device);
  reduce_bf16_kernel<<<blocks, threads, 0, cur_stream()>>>(p.part, p.splits, M, N, M, N,
                                                           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                           static_cast<int>(out.stride(0)), pub);
  TT_CUDA_CHECK(cudaGetLastError());
}

// Grouped SwiGLU experts for decode: act[r] = silu(x_r Wg_e^T) * (x_r Wu_e^T) for the
// token rows r of each expert segment (unpadded segments, grp_off on the device; rows
// at or past grp_off[E] are not computed).  w_gu = [Wg of all E experts; Wu of all E].
void moe_skinny_swiglu_op(torch::Tensor xr, torch::Tensor w_gu, torch::Tensor grp_off, int64_t E, torch::Tensor act) {
  using namespace skinny;
  check_operand(xr, "xr");
  check_operand(w_gu, "w_gu");
  check_cuda_bf16(act, "act");
  const int cap = static_cast<int>(xr.size(0)), K = static_cast<int>(xr.size(1));
  const int I = static_cast<int>(act.size(1));
  TT_CHECK(grp_off.is_cuda() && grp_off.scalar_type() == torch::kInt32 && grp_off.numel() >= E + 1,
           "moe_skinny_swiglu: grp_off int32 [E + 1]");
  TT_CHECK(w_gu.size(0) == 2 * E * I && w_gu.size(1) == K && I % 4 == 0, "moe_skinny_swiglu: w_gu [2*E*I, K]");
  // the split-sum kernel stores 4 bf16 (8 bytes) at a time
  TT_CHECK(act.size(0) == cap && act.stride(1) == 1 && act.stride(0) % 4 == 0 &&
               reinterpret_cast<uintptr_t>(act.data_ptr()) % 8 == 0,
           "moe_skinny_swiglu: act [cap, I], 8-byte aligned");
  check_device(w_gu, xr.get_device(), "moe_skinny_swiglu w_gu");
  check_device(grp_off, xr.get_device(), "moe_skinny_swiglu grp_off");
  check_device(act, xr.get_device(), "moe_skinny_swiglu act");
  if (cap == 0 || E == 0) return;
  const c10::cuda::CUDAGuard guard(xr.device());
  const int device = xr.get_device();
  Params p = base_params(K, device);
  p.n_groups = static_cast<int>(E);
  p.grp_off = grp_off.data_ptr<int>();
  p.halves = 2;
  p.half_cols = I;
  p.half_base0 = 0;
  p.half_base1 = static_cast<int>(E * I);
  p.group_stride = I;
  p.nrb = (I + BW - 1) / BW;
  choose_splits(p, device);
  torch::Tensor part = torch::empty({p.splits, cap, 2 * I}, xr.options().dtype(torch::kFloat32));
  p.part = part.data_ptr<float>();
  p.rows_cap = cap;
  p.ld_part = 2 * I;
  launch(w_gu, xr, p, device);
  const int threads = 256;
  const int blocks = std::max(1, std::min(num_sms(device) * 4, (cap * I / 4 + threads - 1) / threads));
  reduce_swiglu_kernel<<<blocks, threads, 0, cur_stream()>>>(p.part, p.splits, cap, I, p.grp_off + E,
                                                             reinterpret_cast<__nv_bfloat16*>(act.data_ptr()),
                                                             static_cast<int>(act.stride(0)));
  TT_CUDA_CHECK(cudaGetLastError());
}

// Grouped down projection fused with the top-k combine for decode:
// out[n] = sum_j w[n, j] * (act_{slot[n, j]} Wd_e^T), skipping pairs whose slot is at or
// past *row_limit (experts held by other ranks).  wd = [Wd of all E experts] ([E*H, I]).
void moe_skinny_down_combine_op(torch::Tensor act, torch::Tensor wd, torch::Tensor grp_off, int64_t E,
                                torch::Tensor slot, c10::optional<torch::Tensor> w, int64_t k, torch::Tensor out,
                                c10::optional<torch::Tensor> row_limit, int64_t publish_gid, int64_t slot_off,
                                int64_t slot_bytes) {
  using namespace skinny;
  check_operand(act, "act");
  check_operand(wd, "wd");
  check_cuda_bf16(out, "out");
  const int cap = static_cast<int>(act.size(0)), I = static_cast<int>(act.size(1));
  const int N = static_cast<int>(out.size(0)), H = static_cast<int>(out.size(1));
  TT_CHECK(grp_off.is_cuda() && grp_off.scalar_type() == torch::kInt32 && grp_off.numel() >= E + 1,
           "moe_skinny_down: grp_off int32 [E + 1]");
  TT_CHECK(wd.size(0) == E * H && wd.size(1) == I && H % 4 == 0, "moe_skinny_down: wd [E*H, I]");
  TT_CHECK(slot.is_cuda() && slot.scalar_type() == torch::kInt32 && slot.is_contiguous() && slot.numel() == N * k,
           "moe_skinny_down: slot int32 [N * k]");
  if (w.has_value())
    TT_CHECK(w->is_cuda() && w->scalar_type() == torch::kFloat32 && w->is_contiguous() && w->numel() == N * k,
             "moe_skinny_down: w fp32 [N * k]");
  if (row_limit.has_value())
    TT_CHECK(row_limit->is_cuda() && row_limit->scalar_type() == torch::kInt32, "moe_skinny_down: row_limit int32");
  TT_CHECK(out.stride(1) == 1 && out.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 8 == 0,
           "moe_skinny_down: out [N, H], 8-byte aligned");
  const int dev0 = act.get_device();
  check_device(wd, dev0, "moe_skinny_down wd");
  check_device(grp_off, dev0, "moe_skinny_down grp_off");
  check_device(slot, dev0, "moe_skinny_down slot");
  check_device(out, dev0, "moe_skinny_down out");
  if (w.has_value()) check_device(*w, dev0, "moe_skinny_down w");
  if (row_limit.has_value()) check_device(*row_limit, dev0, "moe_skinny_down row_limit");
  if (N == 0) return;
  const c10::cuda::CUDAGuard guard(act.device());
  const int device = act.get_device();
  Params p = base_params(I, device);
  p.n_groups = static_cast<int>(E);
  p.grp_off = grp_off.data_ptr<int>();
  p.halves = 1;
  p.half_cols = H;
  p.half_base0 = p.half_base1 = 0;
  p.group_stride = H;
  p.nrb = (H + BW - 1) / BW;
  choose_splits(p, device);
  torch::Tensor part = torch::empty({p.splits, std::max(cap, 1), H}, act.options().dtype(torch::kFloat32));
  p.part = part.data_ptr<float>();
  p.rows_cap = std::max(cap, 1);
  p.ld_part = H;
  if (cap > 0) launch(wd, act, p, device);
  const Publish pub = make_publish(publish_gid, slot_off, slot_bytes, static_cast<int64_t>(N) * H * 2, device);
  reduce_combine_kernel<<<N, std::min(256, std::max(32, H / 4)), 0, cur_stream()>>>(
      p.part, p.splits, p.rows_cap, H, slot.data_ptr<int>(), w.has_value() ? w->data_ptr<float>() : nullptr,
      static_cast<int>(k), row_limit.has_value() ? row_limit->data_ptr<int>() : p.grp_off + E,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), static_cast<int>(out.stride(0)), pub);
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
