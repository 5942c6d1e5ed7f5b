// MoE routing and token movement on the device (no host synchronisation).
//
// Replaces the reference's router top-k/softmax, token replication, sort / bincount
// and unpermute + weighted sum (tinytron/model/modules/mlp.py:147-161, 240-297):
//   topk_softmax     : per token, the k largest router logits (descending) and the
//                      softmax over them, one warp per token.
//   layout           : expert segments of the grouped GEMMs.  Each expert's rows
//                      start on a multiple of 128 or 256 (pad rows are zero), (token, j)
//                      pairs keep token order inside an expert (stable, so results
//                      do not depend on atomics).  Writes grp_off[E+1], the padded
//                      row of every pair (slot) and the pair of every row (row_pair).
//   gather_rows      : x_rows[r] = x[token of row r] (zeros for pad rows).
//   combine          : out[t] = sum_j w[t,j] * y_rows[slot[t,j]]  (fp32 sum, bf16 out);
//                      without w it is the backward of gather_rows.
//   combine_bwd      : dy_rows[r] = w[pair] * dout[t];  dw[pair] = <dout[t], y_rows[r]>.
//   topk_softmax_bwd : dlogits from dw through the top-k softmax.
#include "common/host_utils.h"
#include "common/ptx.cuh"

namespace tt {
namespace moe {

constexpr int kMaxExperts = 256;
constexpr int kRowAlign = 128;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// One warp per token.  Ties resolve to the lower expert index.
template <typename T>
__global__ void topk_softmax_kernel(const T* __restrict__ logits, int N, int E, int k, float* __restrict__ w,
                                    int* __restrict__ sel) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= N) return;
  constexpr int PER = kMaxExperts / 32;
  float v[PER];
  const T* row = logits + static_cast<size_t>(warp) * E;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    v[i] = (e < E) ? to_f(row[e]) : -INFINITY;
  }
  float top0 = 0.0f, sum = 0.0f;
  float mine = 0.0f;  // lane j < k keeps the j-th value
  int mine_idx = 0;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      if (e < E && (v[i] > best || (v[i] == best && e < bi))) {
        best = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i * 32 + lane == bi) v[i] = -INFINITY;
    if (j == 0) top0 = best;
    const float ex = expf(best - top0);
    sum += ex;
    if (lane == j) {
      mine = ex;
      mine_idx = bi;
    }
  }
  if (lane < k) {
    w[static_cast<size_t>(warp) * k + lane] = mine / sum;
    sel[static_cast<size_t>(warp) * k + lane] = mine_idx;
  }
}

// dlogits[t, :] = 0 except dlogits[t, sel[t,j]] = w_j * (dw_j - sum_i w_i dw_i).
template <typename T>
__global__ void topk_softmax_bwd_kernel(const float* __restrict__ dw, const float* __restrict__ w,
                                        const int* __restrict__ sel, int N, int E, int k, T* __restrict__ dlogits) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= N) return;
  const size_t base = static_cast<size_t>(warp) * k;
  float wj = 0.0f, dj = 0.0f;
  int ej = -1;
  if (lane < k) {
    wj = w[base + lane];
    dj = dw[base + lane];
    ej = sel[base + lane];
  }
  float s = wj * dj;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const float g = wj * (dj - s);
  T* row = dlogits + static_cast<size_t>(warp) * E;
  for (int e = lane; e < E; e += 32) {
    float val = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int ej_b = __shfl_sync(0xffffffffu, ej, j);
      const float gj_b = __shfl_sync(0xffffffffu, g, j);
      if (ej_b == e) val += gj_b;
    }
    if constexpr (sizeof(T) == 4) row[e] = val;
    else row[e] = __float2bfloat16_rn(val);
  }
}

// Expert id of pair i: sel[i], or with remap_lo >= 0 the local id sel[i] - remap_lo when
// that lies in [0, E - 1) and E - 1 (the "remote" group of pairs another rank computes)
// otherwise (expert-parallel inference).
__device__ __forceinline__ int layout_id(const int* __restrict__ sel, int i, int E, int remap_lo) {
  const int x = sel[i];
  if (remap_lo < 0) return x;
  const int l = x - remap_lo;
  return (l >= 0 && l < E - 1) ? l : E - 1;
}

// Grid: one block per expert (1024 threads).  Every block builds the full histogram
// (cheap: the pair list is a few hundred KB and stays in L2), so all offsets are known
// without a second launch; block e then places its own pairs in token order.
__global__ void __launch_bounds__(1024) layout_kernel(const int* __restrict__ sel, int P, int E, int align,
                                                     int* __restrict__ grp_off, int* __restrict__ slot,
                                                     int* __restrict__ row_pair, int* __restrict__ status,
                                                     int remap_lo) {
  __shared__ int hist[kMaxExperts];
  __shared__ int off[kMaxExperts + 1];
  __shared__ int warp_cnt[32];
  __shared__ int running;
  const int e = blockIdx.x;
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int x = layout_id(sel, i, E, remap_lo);
    if (x >= 0 && x < E) atomicAdd(&hist[x], 1);
    else if (e == 0) atomicCAS(status, 0, static_cast<int>(kBadIndex));  // out-of-range expert id: pair dropped
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < E; ++i) {
      off[i] = acc;
      acc += (hist[i] + align - 1) / align * align;
    }
    off[E] = acc;
    running = 0;
  }
  __syncthreads();
  if (e == 0)
    for (int i = threadIdx.x; i <= E; i += blockDim.x) grp_off[i] = off[i];
  const int base = off[e];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int c0 = 0; c0 < P; c0 += blockDim.x) {
    const int i = c0 + threadIdx.x;
    const bool mine = i < P && layout_id(sel, i, E, remap_lo) == e;
    const unsigned bal = __ballot_sync(0xffffffffu, mine);
    if (lane == 0) warp_cnt[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w2 = 0; w2 < nwarps; ++w2) {
      const int c = warp_cnt[w2];
      before += (w2 < warp) ? c : 0;
      total += c;
    }
    if (mine) {
      const int r = base + running + before + __popc(bal & ((1u << lane) - 1u));
      slot[i] = r;
      row_pair[r] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) running += total;
    __syncthreads();
  }
  for (int r = base + hist[e] + threadIdx.x; r < off[e + 1]; r += blockDim.x) row_pair[r] = -1;
}

// The same layout for large pair counts (prefill, training micro-batches) in three
// launches that use the whole GPU instead of one block per expert scanning every pair:
//   1. layout_count_kernel: block b counts the experts of pairs [b*C, (b+1)*C) (shared
//      histogram);
//   2. layout_scan_kernel (one block, a thread per expert): the expert totals, the
//      aligned segment starts (grp_off), each chunk's first row within every expert
//      segment, and the padding rows' row_pair = -1;
//   3. layout_place_kernel: block b walks its chunk 256 pairs at a time; a pair's row is
//      its expert's running count + the same-expert pairs of earlier warps (per-warp
//      counts from __match_any_sync) + its rank among equal lanes of its own warp.
// Rows keep token order within each expert (stable), exactly as the one-block kernel.
constexpr int kLayoutChunk = 4096;
constexpr int kLayoutThreads = 256;

__global__ void __launch_bounds__(kLayoutThreads) layout_count_kernel(const int* __restrict__ sel, int P, int E,
                                                                      int* __restrict__ cnt, int* __restrict__ status,
                                                                      int remap_lo) {
  __shared__ int hist[kMaxExperts];
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int i0 = blockIdx.x * kLayoutChunk, i1 = min(P, i0 + kLayoutChunk);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int x = layout_id(sel, i, E, remap_lo);
    if (x >= 0 && x < E) atomicAdd(&hist[x], 1);
    else atomicCAS(status, 0, static_cast<int>(kBadIndex));  // out-of-range expert id: pair dropped
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[static_cast<size_t>(blockIdx.x) * E + e] = hist[e];
}

__global__ void __launch_bounds__(kMaxExperts) layout_scan_kernel(const int* __restrict__ cnt, int nb, int E,
                                                                  int align, int* __restrict__ grp_off,
                                                                  int* __restrict__ blk_off,
                                                                  int* __restrict__ row_pair) {
  __shared__ int seg[kMaxExperts];
  const int e = threadIdx.x;
  int total = 0;
  if (e < E)
    for (int b = 0; b < nb; ++b) total += cnt[static_cast<size_t>(b) * E + e];
  seg[e] = e < E ? (total + align - 1) / align * align : 0;
  __syncthreads();
  // inclusive scan of the padded segment sizes (Hillis-Steele over kMaxExperts entries)
  for (int d = 1; d < kMaxExperts; d <<= 1) {
    const int v = e >= d ? seg[e - d] : 0;
    __syncthreads();
    seg[e] += v;
    __syncthreads();
  }
  if (e < E) {
    const int start = seg[e] - (total + align - 1) / align * align;
    grp_off[e] = start;
    if (e == E - 1) grp_off[E] = seg[e];
    int run = start;
    for (int b = 0; b < nb; ++b) {
      blk_off[static_cast<size_t>(b) * E + e] = run;
      run += cnt[static_cast<size_t>(b) * E + e];
    }
    for (int r = start + total; r < seg[e]; ++r) row_pair[r] = -1;
  }
}

__global__ void __launch_bounds__(kLayoutThreads) layout_place_kernel(const int* __restrict__ sel, int P, int E,
                                                                      const int* __restrict__ blk_off,
                                                                      int* __restrict__ slot,
                                                                      int* __restrict__ row_pair, int remap_lo) {
  constexpr int NW = kLayoutThreads / 32;
  __shared__ int running[kMaxExperts];
  __shared__ int wcnt[NW][kMaxExperts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) running[e] = blk_off[static_cast<size_t>(blockIdx.x) * E + e];
  const int i0 = blockIdx.x * kLayoutChunk, i1 = min(P, i0 + kLayoutChunk);
  for (int c0 = i0; c0 < i1; c0 += kLayoutThreads) {
    for (int j = threadIdx.x; j < NW * E; j += blockDim.x) wcnt[j / E][j % E] = 0;
    __syncthreads();
    const int i = c0 + threadIdx.x;
    const int x = i < i1 ? layout_id(sel, i, E, remap_lo) : -1;
    const bool ok = x >= 0 && x < E;
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? x : -1);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (ok && rank == 0) wcnt[warp][x] = __popc(peers);
    __syncthreads();
    if (ok) {
      int r = running[x] + rank;
      for (int w = 0; w < warp; ++w) r += wcnt[w][x];
      slot[i] = r;
      row_pair[r] = i;
    } else if (i < i1) {
      slot[i] = -1;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int add = 0;
#pragma unroll
      for (int w = 0; w < NW; ++w) add += wcnt[w][e];
      running[e] += add;
    }
    __syncthreads();
  }
}

// One warp per padded row; rows at or past the device-side total are skipped.
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, int ld_x, const int* __restrict__ row_pair,
                                   const int* __restrict__ total_ptr, int k, int cap, int H,
                                   __nv_bfloat16* __restrict__ out) {
  const int total = *total_ptr;
  const int nvec = H / 8;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < min(total, cap);
       r += (gridDim.x * blockDim.x) >> 5) {
    const int pr = row_pair[r];
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * H);
    if (pr < 0) {
      for (int v = threadIdx.x & 31; v < nvec; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(pr / k) * ld_x);
      for (int v = threadIdx.x & 31; v < nvec; v += 32) dst[v] = src[v];
    }
  }
}

// One block per token, 8 bf16 per thread per step.
// row_limit (optional, device): pairs whose row is at or past *row_limit are skipped (the
// pairs routed to experts on other ranks in expert-parallel inference, whose rows the
// grouped GEMMs never computed); a token with no remaining pair gets zeros.
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y_rows, const int* __restrict__ slot,
                               const float* __restrict__ w, int k, int H, __nv_bfloat16* __restrict__ out,
                               int ld_out, const int* __restrict__ row_limit) {
  const int t = blockIdx.x;
  __shared__ int s_slot[kMaxExperts];
  __shared__ float s_w[kMaxExperts];
  __shared__ int s_k;
  if (threadIdx.x == 0) {  // compact the pairs this rank computed, keeping their order
    const int lim = row_limit ? *row_limit : 0x7fffffff;
    int kk = 0;
    for (int j = 0; j < k; ++j) {
      const int sl = slot[static_cast<size_t>(t) * k + j];
      if (sl >= 0 && sl < lim) {
        s_slot[kk] = sl;
        s_w[kk] = w ? w[static_cast<size_t>(t) * k + j] : 1.0f;
        ++kk;
      }
    }
    s_k = kk;
  }
  __syncthreads();
  const int kk = s_k;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < kk; ++j) {
      const uint4 q = reinterpret_cast<const uint4*>(y_rows + static_cast<size_t>(s_slot[j]) * H)[v];
      const float wj = s_w[j];
      const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(u[i]);
        acc[2 * i] = fmaf(wj, f.x, acc[2 * i]);
        acc[2 * i + 1] = fmaf(wj, f.y, acc[2 * i + 1]);
      }
    }
    reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * ld_out)[v] =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
}

// One warp per padded row.
__global__ void combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout, int ld_dout,
                                   const __nv_bfloat16* __restrict__ y_rows, const int* __restrict__ row_pair,
                                   const float* __restrict__ w, const int* __restrict__ total_ptr, int k, int cap,
                                   int H, __nv_bfloat16* __restrict__ dy_rows, float* __restrict__ dw) {
  const int total = *total_ptr;
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < min(total, cap);
       r += (gridDim.x * blockDim.x) >> 5) {
    const int pr = row_pair[r];
    uint4* dst = reinterpret_cast<uint4*>(dy_rows + static_cast<size_t>(r) * H);
    if (pr < 0) {
      for (int v = lane; v < nvec; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const float wp = w[pr];
    const uint4* g = reinterpret_cast<const uint4*>(dout + static_cast<size_t>(pr / k) * ld_dout);
    const uint4* y = reinterpret_cast<const uint4*>(y_rows + static_cast<size_t>(r) * H);
    float dot = 0.0f;
    for (int v = lane; v < nvec; v += 32) {
      const uint4 gq = g[v], yq = y[v];
      const uint32_t gu[4] = {gq.x, gq.y, gq.z, gq.w}, yu[4] = {yq.x, yq.y, yq.z, yq.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 gf = unpack_bf16x2(gu[i]), yf = unpack_bf16x2(yu[i]);
        dot = fmaf(gf.x, yf.x, fmaf(gf.y, yf.y, dot));
        o[i] = pack_bf16x2(wp * gf.x, wp * gf.y);
      }
      dst[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    if (lane == 0) dw[pr] = dot;
  }
}

static int row_blocks(int rows, int device) {
  return std::max(1, std::min((rows + 7) / 8, num_sms(device) * 8));
}

}  // namespace moe

// ---------------------------------------------------------------------------- host
void moe_topk_softmax_op(torch::Tensor logits, int64_t k, torch::Tensor w, torch::Tensor sel) {
  TT_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(), "topk: logits must be contiguous [N, E]");
  const int N = static_cast<int>(logits.size(0)), E = static_cast<int>(logits.size(1));
  TT_CHECK(E <= moe::kMaxExperts && k >= 1 && k <= 32 && k <= E, "topk: E <= 256, 1 <= k <= min(32, E)");
  TT_CHECK(w.scalar_type() == torch::kFloat32 && sel.scalar_type() == torch::kInt32 && w.numel() == N * k &&
               sel.numel() == N * k && w.is_contiguous() && sel.is_contiguous(), "topk: bad outputs");
  if (N == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  const int blocks = (N + 7) / 8;
  if (logits.scalar_type() == torch::kFloat32)
    moe::topk_softmax_kernel<float><<<blocks, 256, 0, cur_stream()>>>(logits.data_ptr<float>(), N, E,
                                                                       static_cast<int>(k), w.data_ptr<float>(),
                                                                       sel.data_ptr<int>());
  else {
    TT_CHECK(logits.scalar_type() == torch::kBFloat16, "topk: logits fp32 or bf16");
    moe::topk_softmax_kernel<__nv_bfloat16><<<blocks, 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), N, E, static_cast<int>(k), w.data_ptr<float>(),
        sel.data_ptr<int>());
  }
  TT_CUDA_CHECK(cudaGetLastError());
}

void moe_topk_softmax_bwd_op(torch::Tensor dw, torch::Tensor w, torch::Tensor sel, torch::Tensor dlogits) {
  TT_CHECK(dlogits.is_cuda() && dlogits.dim() == 2 && dlogits.is_contiguous(), "topk_bwd: dlogits [N, E]");
  const int N = static_cast<int>(dlogits.size(0)), E = static_cast<int>(dlogits.size(1));
  const int k = static_cast<int>(w.numel() / std::max(N, 1));
  TT_CHECK(dw.is_contiguous() && w.is_contiguous() && sel.is_contiguous() && dw.numel() == w.numel() &&
               sel.numel() == w.numel() && k <= 32 && dw.scalar_type() == torch::kFloat32 &&
               sel.scalar_type() == torch::kInt32, "topk_bwd: bad inputs");
  if (N == 0) return;
  const c10::cuda::CUDAGuard guard(dlogits.device());
  const int blocks = (N + 7) / 8;
  if (dlogits.scalar_type() == torch::kFloat32)
    moe::topk_softmax_bwd_kernel<float><<<blocks, 256, 0, cur_stream()>>>(
        dw.data_ptr<float>(), w.data_ptr<float>(), sel.data_ptr<int>(), N, E, k, dlogits.data_ptr<float>());
  else
    moe::topk_softmax_bwd_kernel<__nv_bfloat16><<<blocks, 256, 0, cur_stream()>>>(
        dw.data_ptr<float>(), w.data_ptr<float>(), sel.data_ptr<int>(), N, E, k,
        reinterpret_cast<__nv_bfloat16*>(dlogits.data_ptr()));
  TT_CUDA_CHECK(cudaGetLastError());
}

// Capacity of the padded row space for P pairs over E experts, segments aligned to
// `align` rows (128, or 256 for the CTA-pair grouped GEMM whose tiles span 256 rows; 1 for
// the unpadded segments of the decode-sized weight-streaming path).
int64_t moe_row_capacity(int64_t P, int64_t E, int64_t align) {
  TT_CHECK(align == 1 || align == 128 || align == 256, "moe: segment alignment must be 1, 128 or 256");
  return (P + E * (align - 1) + align - 1) / align * align;
}

void moe_layout_op(torch::Tensor sel, int64_t E, torch::Tensor grp_off, torch::Tensor slot, torch::Tensor row_pair,
                   int64_t align, int64_t remap_lo) {
  TT_CHECK(sel.is_cuda() && sel.scalar_type() == torch::kInt32 && sel.is_contiguous(), "layout: sel int32");
  const int P = static_cast<int>(sel.numel());
  TT_CHECK(E >= 1 && E <= moe::kMaxExperts, "layout: 1 <= E <= 256");
  TT_CHECK(grp_off.scalar_type() == torch::kInt32 && grp_off.numel() == E + 1 && slot.numel() == P &&
               slot.scalar_type() == torch::kInt32 && row_pair.scalar_type() == torch::kInt32 &&
               row_pair.numel() >= moe_row_capacity(P, E, align), "layout: bad outputs");
  const c10::cuda::CUDAGuard guard(sel.device());
  int* status = device_status_ptr(sel.get_device());
  if (P <= 2 * moe::kLayoutChunk) {  // decode and small batches: one launch
    moe::layout_kernel<<<static_cast<unsigned>(E), 1024, 0, cur_stream()>>>(
        sel.data_ptr<int>(), P, static_cast<int>(E), static_cast<int>(align), grp_off.data_ptr<int>(),
        slot.data_ptr<int>(), row_pair.data_ptr<int>(), status, static_cast<int>(remap_lo));
    TT_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int nb = (P + moe::kLayoutChunk - 1) / moe::kLayoutChunk;
  torch::Tensor scratch = torch::empty({2, nb, E}, sel.options());
  int* cnt = scratch.data_ptr<int>();
  int* blk_off = cnt + static_cast<size_t>(nb) * E;
  moe::layout_count_kernel<<<nb, moe::kLayoutThreads, 0, cur_stream()>>>(sel.data_ptr<int>(), P, static_cast<int>(E),
                                                                         cnt, status, static_cast<int>(remap_lo));
  moe::layout_scan_kernel<<<1, moe::kMaxExperts, 0, cur_stream()>>>(cnt, nb, static_cast<int>(E),
                                                                    static_cast<int>(align), grp_off.data_ptr<int>(),
                                                                    blk_off, row_pair.data_ptr<int>());
  moe::layout_place_kernel<<<nb, moe::kLayoutThreads, 0, cur_stream()>>>(
      sel.data_ptr<int>(), P, static_cast<int>(E), blk_off, slot.data_ptr<int>(), row_pair.data_ptr<int>(),
      static_cast<int>(remap_lo));
  TT_CUDA_CHECK(cudaGetLastError());
}

void moe_gather_rows_op(torch::Tensor x, torch::Tensor row_pair, torch::Tensor grp_off, int64_t k, torch::Tensor out) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(out, "out");
  const int H = static_cast<int>(x.size(1));
  TT_CHECK(H % 8 == 0 && x.stride(1) == 1 && x.stride(0) % 8 == 0 && out.is_contiguous() && out.size(1) == H,
           "gather_rows: bad shapes");
  const int cap = static_cast<int>(out.size(0));
  TT_CHECK(row_pair.numel() >= cap, "gather_rows: row_pair too short");
  const int E = static_cast<int>(grp_off.numel() - 1);
  const c10::cuda::CUDAGuard guard(x.device());
  moe::gather_rows_kernel<<<moe::row_blocks(cap, x.get_device()), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), static_cast<int>(x.stride(0)), row_pair.data_ptr<int>(),
      grp_off.data_ptr<int>() + E, static_cast<int>(k), cap, H, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  TT_CUDA_CHECK(cudaGetLastError());
}

void moe_combine_op(torch::Tensor y_rows, torch::Tensor slot, c10::optional<torch::Tensor> w, int64_t k,
                    torch::Tensor out, c10::optional<torch::Tensor> row_limit) {
  check_cuda_bf16(y_rows, "y_rows");
  check_cuda_bf16(out, "out");
  const int H = static_cast<int>(y_rows.size(1));
  const int N = static_cast<int>(out.size(0));
  TT_CHECK(k >= 1 && k <= moe::kMaxExperts && H % 8 == 0 && y_rows.is_contiguous() && out.size(1) == H &&
               out.stride(1) == 1 && out.stride(0) % 8 == 0 && slot.numel() == N * k, "combine: bad shapes");
  if (w.has_value()) TT_CHECK(w->scalar_type() == torch::kFloat32 && w->numel() == N * k, "combine: w fp32 [N, k]");
  if (row_limit.has_value())
    TT_CHECK(row_limit->is_cuda() && row_limit->scalar_type() == torch::kInt32 && row_limit->numel() >= 1,
             "combine: row_limit int32 device scalar");
  if (N == 0) return;
  const c10::cuda::CUDAGuard guard(out.device());
  moe::combine_kernel<<<static_cast<unsigned>(N), std::min(256, std::max(32, H / 8)), 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y_rows.data_ptr()), slot.data_ptr<int>(),
      w.has_value() ? w->data_ptr<float>() : nullptr, static_cast<int>(k), H,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), static_cast<int>(out.stride(0)),
      row_limit.has_value() ? row_limit->data_ptr<int>() : nullptr);
  TT_CUDA_CHECK(cudaGetLastError());
}

void moe_combine_bwd_op(torch::Tensor dout, torch::Tensor y_rows, torch::Tensor row_pair, torch::Tensor w,
                        torch::Tensor grp_off, int64_t k, torch::Tensor dy_rows, torch::Tensor dw) {
  check_cuda_bf16(dout, "dout");
  check_cuda_bf16(y_rows, "y_rows");
  check_cuda_bf16(dy_rows, "dy_rows");
  const int H = static_cast<int>(y_rows.size(1));
  const int cap = static_cast<int>(y_rows.size(0));
  TT_CHECK(dy_rows.size(0) == cap && dy_rows.is_contiguous() && y_rows.is_contiguous() && H % 8 == 0 &&
               dout.stride(1) == 1 && dout.stride(0) % 8 == 0 && dw.scalar_type() == torch::kFloat32 &&
               w.scalar_type() == torch::kFloat32 && dw.numel() == w.numel(), "combine_bwd: bad shapes");
  const int E = static_cast<int>(grp_off.numel() - 1);
  const c10::cuda::CUDAGuard guard(dout.device());
  moe::combine_bwd_kernel<<<moe::row_blocks(cap, dout.get_device()), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), static_cast<int>(dout.stride(0)),
      reinterpret_cast<const __nv_bfloat16*>(y_rows.data_ptr()), row_pair.data_ptr<int>(), w.data_ptr<float>(),
      grp_off.data_ptr<int>() + E, static_cast<int>(k), cap, H, reinterpret_cast<__nv_bfloat16*>(dy_rows.data_ptr()),
      dw.data_ptr<float>());
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
