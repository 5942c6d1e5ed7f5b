// Expert-parallel dispatch and combine over NVLink peer memory (symmetric heap of
// csrc/runtime/comm.cu).  Replaces the reference's EP all-to-alls
// (tinytron/distributed/expert_parallel/comm.py:22-164, model/modules/mlp.py:257-293):
//
//   * allgather_counts  every rank stores its per-expert send counts [E] into row
//                       `rank` of every peer's count matrix [world, E] (one small
//                       kernel, bounded wait); the host then knows every segment size.
//   * scatter           a warp per (token, slot) pair stores the token's hidden row
//                       straight into the owning rank's expert-grouped receive buffer
//                       at a precomputed row (P2P stores; no sort-then-a2a copies).
//                       The backward variant stores w * dout[token] and also computes
//                       dw = <dout[token], y_pair> for the router weights.
//   * pull_combine      a warp per token loads its k expert outputs from the owning
//                       ranks' output buffers (P2P loads), optionally keeps them (for
//                       the backward), and writes sum_j w_j * y_j (fp32 accumulate).
//   * zero_pad          zeroes the padding rows of the 128-row-aligned expert segments
//                       of the local receive buffer (the grouped GEMMs read them).
//   * fused combine     (push instead of pull) the forward scatter also stores, per
//                       received row, where its expert output must go: the sender's rank
//                       and the byte offset of slot `pair` in the sender's return buffer.
//                       resolve_rows turns those into addresses in this process (peer
//                       pointers) for the down-projection GEMM, whose epilogue then stores
//                       every output row straight into the sender's memory; after one
//                       barrier the sender sums its k rows locally (local_combine).
//
// Every launch records a bad index (row beyond the buffer, rank beyond the group)
// in the device status word and skips that row instead of faulting.
#include "runtime/comm_common.cuh"

namespace tt {
namespace ep {

using comm::PeerTable;

constexpr int kThreads = 256;  // 8 warps per block, one pair / token per warp

__global__ void allgather_kernel(PeerTable t, const int* __restrict__ src, int n, size_t dst_off, uint64_t e,
                                 int* status, uint64_t timeout_ns) {
  for (int p = 0; p < t.world; ++p) {
    int* dst = reinterpret_cast<int*>(t.base[p] + dst_off) + static_cast<long long>(t.rank) * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    comm::signal_peers(t, e);
    comm::wait_peers(t, e, status, timeout_ns);
  }
}

// MODE 0 (forward): row = x[pair / k].  MODE 1 (backward): row = w[pair] * x[pair / k]
// and dw[pair] = <x[pair / k], y_pair[pair]>.
template <int MODE>
__global__ void __launch_bounds__(kThreads) scatter_kernel(PeerTable t, const __nv_bfloat16* __restrict__ x,
                                                          int num_pairs, int k, int H, const int* __restrict__ tgt,
                                                          const int* __restrict__ dst, long long cap, size_t recv_off,
                                                          const float* __restrict__ w,
                                                          const __nv_bfloat16* __restrict__ y_pairs,
                                                          float* __restrict__ dw, uint64_t e_done, int* status,
                                                          long long ret_off, long long back_off) {
  const int warp = (blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int n_warps = (gridDim.x * kThreads) >> 5;
  const int nv = H / 8;  // uint4 (8 bf16) per row
  for (int pr = warp; pr < num_pairs; pr += n_warps) {
    const int r = tgt[pr];
    const long long row = dst[pr];
    if (r < 0 || r >= t.world || row < 0 || row >= cap) {
      if (lane == 0) atomicCAS(status, 0, static_cast<int>(kBadIndex));
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(pr / k) * H);
    uint4* out = reinterpret_cast<uint4*>(t.base[r] + recv_off + row * H * 2);
    if constexpr (MODE == 0) {
      for (int i = lane; i < nv; i += 32) out[i] = src[i];
      if (ret_off >= 0 && lane == 0) {  // return address: (sender rank, offset of slot pr) + 1
        const unsigned long long v =
            ((static_cast<unsigned long long>(t.rank) << 48) | static_cast<unsigned long long>(back_off + pr * H * 2ll)) + 1ull;
        reinterpret_cast<unsigned long long*>(t.base[r] + ret_off)[row] = v;
      }
    } else {
      const float wv = w[pr];
      const uint4* yp = reinterpret_cast<const uint4*>(y_pairs + static_cast<long long>(pr) * H);
      float dot = 0.f;
      for (int i = lane; i < nv; i += 32) {
        const uint4 a = src[i];
        const uint4 b = yp[i];
        const uint32_t* av = reinterpret_cast<const uint32_t*>(&a);
        const uint32_t* bv = reinterpret_cast<const uint32_t*>(&b);
        uint4 o;
        uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 fa = unpack_bf16x2(av[q]);
          const float2 fb = unpack_bf16x2(bv[q]);
          dot += fa.x * fb.x + fa.y * fb.y;
          ov[q] = pack_bf16x2(wv * fa.x, wv * fa.y);
        }
        out[i] = o;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (lane == 0) dw[pr] = dot;
    }
  }
  comm::grid_last_block(t, [&]() { comm::signal_peers(t, e_done); });
}

// out[tok] = sum_j w[tok*k+j] * peer(tgt).y[dst]  (w == nullptr: plain sum); y_save[pair] = row.
template <int PL>  // uint4 columns per lane: H <= PL * 256
__global__ void __launch_bounds__(kThreads) pull_combine_kernel(PeerTable t, size_t y_off, int N, int k, int H,
                                                               const int* __restrict__ tgt,
                                                               const int* __restrict__ dst, long long cap,
                                                               const float* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ out,
                                                               __nv_bfloat16* __restrict__ y_save, int* status,
                                                               int local) {
  const int warp = (blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int n_warps = (gridDim.x * kThreads) >> 5;
  const int nv = H / 8;
  for (int tok = warp; tok < N; tok += n_warps) {
    // Each lane accumulates its uint4 columns over the k slots.
    float acc[PL][8];
#pragma unroll
    for (int c = 0; c < PL; ++c)
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[c][q] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int pr = tok * k + j;
      const int r = local ? t.rank : tgt[pr];        // local: rows were pushed into slot `pr` here
      const long long row = local ? pr : dst[pr];
      if (r < 0 || r >= t.world || row < 0 || row >= cap) {
        if (lane == 0) atomicCAS(status, 0, static_cast<int>(kBadIndex));
        continue;
      }
      const float wv = w != nullptr ? w[pr] : 1.0f;
      const uint4* src = reinterpret_cast<const uint4*>(t.base[r] + y_off + row * H * 2);
      uint4* save = y_save != nullptr ? reinterpret_cast<uint4*>(y_save + static_cast<long long>(pr) * H) : nullptr;
#pragma unroll
      for (int c = 0; c < PL; ++c) {
        const int i = lane + 32 * c;
        if (i < nv) {
          const uint4 v = src[i];
          if (save != nullptr) save[i] = v;
          const uint32_t* vv = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(vv[q]);
            acc[c][2 * q] += wv * f.x;
            acc[c][2 * q + 1] += wv * f.y;
          }
        }
      }
    }
    uint4* o = reinterpret_cast<uint4*>(out + static_cast<long long>(tok) * H);
#pragma unroll
    for (int c = 0; c < PL; ++c) {
      const int i = lane + 32 * c;
      if (i < nv) {
        uint4 u;
        uint32_t* uv = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) uv[q] = pack_bf16x2(acc[c][2 * q], acc[c][2 * q + 1]);
        o[i] = u;
      }
    }
  }
}

// row_ptr[r] = address (in this process) of the return slot recorded for received row r,
// 0 for rows nobody sent (segment padding); the record is cleared for the next exchange.
__global__ void resolve_rows_kernel(PeerTable t, long long ret_off, int rows, int H, long long heap_bytes,
                                    long long* __restrict__ row_ptr, int* status) {
  unsigned long long* ret = reinterpret_cast<unsigned long long*>(t.base[t.rank] + ret_off);
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const unsigned long long v = ret[r];
    long long a = 0;
    if (v != 0ull) {
      const int src = static_cast<int>((v - 1ull) >> 48);
      const long long off = static_cast<long long>((v - 1ull) & ((1ull << 48) - 1ull));
      if (src < t.world && off >= 0 && off + 2ll * H <= heap_bytes) {
        a = reinterpret_cast<long long>(t.base[src] + off);
      } else {
        atomicCAS(status, 0, static_cast<int>(kBadIndex));
      }
      ret[r] = 0ull;
    }
    row_ptr[r] = a;
  }
}

// Zero rows [seg_off[e] + seg_cnt[e], seg_off[e + 1]) of buf [rows, H] for every e.
__global__ void zero_pad_kernel(__nv_bfloat16* __restrict__ buf, const int* __restrict__ seg_off,
                                const int* __restrict__ seg_cnt, int n_seg, int H, long long cap) {
  const int e = blockIdx.y;
  if (e >= n_seg) return;
  const long long r0 = static_cast<long long>(seg_off[e]) + seg_cnt[e];
  const long long r1 = min(static_cast<long long>(seg_off[e + 1]), cap);
  const int nv = H / 8;
  const long long total = (r1 - r0) * nv;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    reinterpret_cast<uint4*>(buf + r0 * H)[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Destination of every (token, slot) pair of this rank: dst = slot + delta[e], tgt = e / E_l,
// where slot is the pair's position in this rank's expert-sorted (stable) order and
// delta[e] = (owner row of expert e's first pair from this rank) - (expert e's first
// position in that order).  Out-of-range expert ids are recorded and sent to row 0 of rank 0.
__global__ void plan_rows_kernel(const int* __restrict__ sel, const int* __restrict__ slot,
                                 const int* __restrict__ delta, int P, int E, int E_l, int* __restrict__ dst,
                                 int* __restrict__ tgt, int* __restrict__ status) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P; i += gridDim.x * blockDim.x) {
    const int e = sel[i];
    if (e < 0 || e >= E) {
      atomicCAS(status, 0, static_cast<int>(kBadIndex));
      dst[i] = 0;
      tgt[i] = 0;
      continue;
    }
    dst[i] = slot[i] + delta[e];
    tgt[i] = e / E_l;
  }
}

}  // namespace ep

namespace {
void check_pairs(const torch::Tensor& tgt, const torch::Tensor& dst, int64_t P) {
  TT_CHECK(tgt.scalar_type() == torch::kInt32 && dst.scalar_type() == torch::kInt32 && tgt.numel() == P &&
               dst.numel() == P && tgt.is_contiguous() && dst.is_contiguous() && tgt.is_cuda() && dst.is_cuda(),
           "ep: tgt/dst must be contiguous CUDA int32 [pairs]");
}
}  // namespace

// Pair destinations from the stable expert order (see plan_rows_kernel).
void ep_plan_rows(torch::Tensor sel, torch::Tensor slot, torch::Tensor delta, int64_t E_l, torch::Tensor dst,
                  torch::Tensor tgt) {
  const int64_t P = sel.numel();
  TT_CHECK(sel.is_cuda() && sel.scalar_type() == torch::kInt32 && sel.is_contiguous() && slot.numel() == P &&
               slot.scalar_type() == torch::kInt32 && slot.is_contiguous() && delta.scalar_type() == torch::kInt32 &&
               delta.is_contiguous(),
           "ep_plan_rows: sel, slot int32 [P], delta int32 [E]");
  check_pairs(tgt, dst, P);
  const int dev = sel.get_device();
  TT_CHECK(slot.is_cuda() && slot.get_device() == dev && delta.is_cuda() && delta.get_device() == dev &&
               dst.get_device() == dev && tgt.get_device() == dev,
           "ep_plan_rows: every operand on sel's device");
  const int64_t E = delta.numel();
  TT_CHECK(E_l >= 1 && E % E_l == 0, "ep_plan_rows: E must be a multiple of E_l");
  if (P == 0) return;
  const c10::cuda::CUDAGuard guard(sel.device());
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>((P + threads - 1) / threads, 4 * num_sms(sel.get_device())));
  ep::plan_rows_kernel<<<blocks, threads, 0, cur_stream()>>>(
      sel.data_ptr<int>(), slot.data_ptr<int>(), delta.data_ptr<int>(), static_cast<int>(P), static_cast<int>(E),
      static_cast<int>(E_l), dst.data_ptr<int>(), tgt.data_ptr<int>(), device_status_ptr(sel.get_device()));
  TT_CUDA_CHECK(cudaGetLastError());
}

// counts int32 [E] -> row `rank` of the [world, E] matrix at heap offset dst_off on every rank.
void ep_allgather_counts(int64_t gid, torch::Tensor counts, int64_t dst_off) {
  TT_CHECK(counts.scalar_type() == torch::kInt32 && counts.is_cuda() && counts.is_contiguous(),
           "ep_allgather_counts: counts must be CUDA int32");
  const comm::PeerTable t = comm::group_table(gid);
  const int64_t n = counts.numel();
  TT_CHECK(dst_off % 16 == 0 && dst_off + t.world * n * 4 <= static_cast<int64_t>(comm::group_bytes(gid)),
           "ep_allgather_counts: destination outside the heap");
  const c10::cuda::CUDAGuard guard(counts.device());
  const bool emu = comm::group_emulated(gid);
  const uint64_t e = emu ? 0ull : comm::group_next_epoch(gid);
  ep::allgather_kernel<<<1, 256, 0, cur_stream()>>>(t, counts.data_ptr<int>(), static_cast<int>(n),
                                                    static_cast<size_t>(dst_off), e,
                                                    device_status_ptr(counts.get_device()), comm::wait_timeout_ns());
  TT_CUDA_CHECK(cudaGetLastError());
}

// Store pair rows into the owners' receive buffers (heap offset recv_off, cap rows of H
// bf16), then wait until every peer finished its own scatter.  Backward mode (w given):
// rows are w[pair] * x[pair / k] and dw[pair] = <x[pair / k], y_pairs[pair]>.
// Forward mode with ret_off >= 0 also records, for every row, its return address
// (this rank, heap offset back_off + pair * H * 2) in the owner's int64 array at ret_off.
void ep_scatter(int64_t gid, torch::Tensor x, int64_t k, torch::Tensor tgt, torch::Tensor dst, int64_t recv_off,
                int64_t cap, c10::optional<torch::Tensor> w, c10::optional<torch::Tensor> y_pairs,
                c10::optional<torch::Tensor> dw, int64_t ret_off, int64_t back_off) {
  check_cuda_bf16(x, "x");
  TT_CHECK(x.dim() == 2 && x.is_contiguous() && x.size(1) % 8 == 0 && x.size(1) <= 4096,
           "ep_scatter: x must be contiguous [N, H], H % 8 == 0, H <= 4096");
  const int64_t N = x.size(0), H = x.size(1), P = N * k;
  check_pairs(tgt, dst, P);
  const comm::PeerTable t = comm::group_table(gid);
  TT_CHECK(recv_off % 256 == 0 && recv_off + cap * H * 2 <= static_cast<int64_t>(comm::group_bytes(gid)),
           "ep_scatter: receive buffer outside the heap");
  const bool bwd = w.has_value();
  if (ret_off >= 0) {
    TT_CHECK(!bwd, "ep_scatter: return addresses are recorded in forward mode only");
    TT_CHECK(ret_off % 8 == 0 && ret_off + cap * 8 <= static_cast<int64_t>(comm::group_bytes(gid)) &&
                 back_off % 16 == 0 && back_off >= 0 && back_off + P * H * 2 <= static_cast<int64_t>(comm::group_bytes(gid)),
             "ep_scatter: return-address array or return buffer outside the heap");
    TT_CHECK(back_off + P * H * 2 < (1ll << 48), "ep_scatter: heap offsets must fit in 48 bits");
  }
  if (bwd) {
    TT_CHECK(y_pairs.has_value() && dw.has_value(), "ep_scatter: backward needs y_pairs and dw");
    TT_CHECK(w->scalar_type() == torch::kFloat32 && w->numel() == P && w->is_contiguous(), "ep_scatter: w fp32 [P]");
    check_cuda_bf16(*y_pairs, "y_pairs");
    TT_CHECK(y_pairs->numel() == P * H && y_pairs->is_contiguous(), "ep_scatter: y_pairs [P, H]");
    TT_CHECK(dw->scalar_type() == torch::kFloat32 && dw->numel() == P, "ep_scatter: dw fp32 [P]");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const int dev = x.get_device();
  const bool emu = comm::group_emulated(gid);
  const uint64_t e = emu ? 0ull : comm::group_next_epoch(gid);
  const int grid = comm::grid_blocks(dev, std::max<int64_t>(1, P * 32), ep::kThreads);
  int* st = device_status_ptr(dev);
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  if (!bwd) {
    ep::scatter_kernel<0><<<grid, ep::kThreads, 0, cur_stream()>>>(
        t, xp, static_cast<int>(P), static_cast<int>(k), static_cast<int>(H), tgt.data_ptr<int>(),
        dst.data_ptr<int>(), cap, static_cast<size_t>(recv_off), nullptr, nullptr, nullptr, e, st, ret_off, back_off);
  } else {
    ep::scatter_kernel<1><<<grid, ep::kThreads, 0, cur_stream()>>>(
        t, xp, static_cast<int>(P), static_cast<int>(k), static_cast<int>(H), tgt.data_ptr<int>(),
        dst.data_ptr<int>(), cap, static_cast<size_t>(recv_off), w->data_ptr<float>(),
        reinterpret_cast<const __nv_bfloat16*>(y_pairs->data_ptr()), dw->data_ptr<float>(), e, st, -1ll, 0ll);
  }
  TT_CUDA_CHECK(cudaGetLastError());
  if (!emu) comm::launch_peer_wait(t, e, st, cur_stream());  // every peer's scatter-done epoch
}

// out[tok] = sum_j w[tok*k+j] * owner(tgt).buffer[dst]  (heap offset y_off); y_save keeps the rows.
void ep_pull_combine(int64_t gid, int64_t y_off, int64_t cap, torch::Tensor tgt, torch::Tensor dst, int64_t k,
                     c10::optional<torch::Tensor> w, torch::Tensor out, c10::optional<torch::Tensor> y_save) {
  check_cuda_bf16(out, "out");
  TT_CHECK(out.dim() == 2 && out.is_contiguous() && out.size(1) % 8 == 0 && out.size(1) <= 4096,
           "ep_pull_combine: out [N, H], H % 8 == 0, H <= 4096");
  const int64_t N = out.size(0), H = out.size(1), P = N * k;
  check_pairs(tgt, dst, P);
  TT_CHECK(y_off % 256 == 0 && y_off + cap * H * 2 <= static_cast<int64_t>(comm::group_bytes(gid)),
           "ep_pull_combine: source buffer outside the heap");
  const float* wp = nullptr;
  if (w.has_value()) {
    TT_CHECK(w->scalar_type() == torch::kFloat32 && w->numel() == P && w->is_contiguous(),
             "ep_pull_combine: w fp32 [P]");
    wp = w->data_ptr<float>();
  }
  __nv_bfloat16* sp = nullptr;
  if (y_save.has_value()) {
    check_cuda_bf16(*y_save, "y_save");
    TT_CHECK(y_save->numel() == P * H && y_save->is_contiguous(), "ep_pull_combine: y_save [P, H]");
    sp = reinterpret_cast<__nv_bfloat16*>(y_save->data_ptr());
  }
  const comm::PeerTable t = comm::group_table(gid);
  const c10::cuda::CUDAGuard guard(out.device());
  const int dev = out.get_device();
  const int grid = comm::grid_blocks(dev, std::max<int64_t>(1, N * 32), ep::kThreads);
  const int pl = static_cast<int>((H / 8 + 31) / 32);
#define TT_PULL(PLV)                                                                                              \
  ep::pull_combine_kernel<PLV><<<grid, ep::kThreads, 0, cur_stream()>>>(                                           \
      t, static_cast<size_t>(y_off), static_cast<int>(N), static_cast<int>(k), static_cast<int>(H),              \
      tgt.data_ptr<int>(), dst.data_ptr<int>(), cap, wp, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), sp, \
      device_status_ptr(dev), 0)
  if (pl <= 2) TT_PULL(2);
  else if (pl <= 4) TT_PULL(4);
  else if (pl <= 8) TT_PULL(8);
  else TT_PULL(16);
#undef TT_PULL
  TT_CUDA_CHECK(cudaGetLastError());
}

// out[tok] = sum_j w[tok*k+j] * buffer[tok*k+j] over this rank's own return buffer (heap
// offset y_off, filled by the owners' down-projection epilogues); y_save keeps the rows.
void ep_local_combine(int64_t gid, int64_t y_off, int64_t k, c10::optional<torch::Tensor> w, torch::Tensor out,
                      c10::optional<torch::Tensor> y_save) {
  check_cuda_bf16(out, "out");
  TT_CHECK(out.dim() == 2 && out.is_contiguous() && out.size(1) % 8 == 0 && out.size(1) <= 4096,
           "ep_local_combine: out [N, H], H % 8 == 0, H <= 4096");
  const int64_t N = out.size(0), H = out.size(1), P = N * k;
  TT_CHECK(y_off % 256 == 0 && y_off + P * H * 2 <= static_cast<int64_t>(comm::group_bytes(gid)),
           "ep_local_combine: return buffer outside the heap");
  const float* wp = nullptr;
  if (w.has_value()) {
    TT_CHECK(w->scalar_type() == torch::kFloat32 && w->numel() == P && w->is_contiguous(),
             "ep_local_combine: w fp32 [P]");
    wp = w->data_ptr<float>();
  }
  __nv_bfloat16* sp = nullptr;
  if (y_save.has_value()) {
    check_cuda_bf16(*y_save, "y_save");
    TT_CHECK(y_save->numel() == P * H && y_save->is_contiguous(), "ep_local_combine: y_save [P, H]");
    sp = reinterpret_cast<__nv_bfloat16*>(y_save->data_ptr());
  }
  const comm::PeerTable t = comm::group_table(gid);
  const c10::cuda::CUDAGuard guard(out.device());
  const int dev = out.get_device();
  const int grid = comm::grid_blocks(dev, std::max<int64_t>(1, N * 32), ep::kThreads);
  const int pl = static_cast<int>((H / 8 + 31) / 32);
#define TT_LOCAL(PLV)                                                                                          \
  ep::pull_combine_kernel<PLV><<<grid, ep::kThreads, 0, cur_stream()>>>(                                        \
      t, static_cast<size_t>(y_off), static_cast<int>(N), static_cast<int>(k), static_cast<int>(H), nullptr, \
      nullptr, P, wp, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), sp, device_status_ptr(dev), 1)
  if (pl <= 2) TT_LOCAL(2);
  else if (pl <= 4) TT_LOCAL(4);
  else if (pl <= 8) TT_LOCAL(8);
  else TT_LOCAL(16);
#undef TT_LOCAL
  TT_CUDA_CHECK(cudaGetLastError());
}

// row_ptr[r] (int64, r < rows) = peer address of the return slot recorded for received row
// r by the forward scatter (heap offset ret_off), 0 for padding rows; clears the records.
void ep_resolve_rows(int64_t gid, int64_t ret_off, int64_t rows, int64_t H, torch::Tensor row_ptr) {
  TT_CHECK(row_ptr.is_cuda() && row_ptr.scalar_type() == torch::kInt64 && row_ptr.is_contiguous() &&
               row_ptr.numel() >= rows,
           "ep_resolve_rows: row_ptr must be a contiguous CUDA int64 tensor of >= rows entries");
  const int64_t bytes = static_cast<int64_t>(comm::group_bytes(gid));
  TT_CHECK(ret_off % 8 == 0 && ret_off + rows * 8 <= bytes, "ep_resolve_rows: record array outside the heap");
  if (rows == 0) return;
  const comm::PeerTable t = comm::group_table(gid);
  const c10::cuda::CUDAGuard guard(row_ptr.device());
  const int dev = row_ptr.get_device();
  const int grid = static_cast<int>(std::min<int64_t>((rows + 255) / 256, 1024));
  ep::resolve_rows_kernel<<<grid, 256, 0, cur_stream()>>>(t, ret_off, static_cast<int>(rows), static_cast<int>(H),
                                                          bytes, reinterpret_cast<long long*>(row_ptr.data_ptr<int64_t>()),
                                                          device_status_ptr(dev));
  TT_CUDA_CHECK(cudaGetLastError());
}

void ep_zero_pad(torch::Tensor buf, torch::Tensor seg_off, torch::Tensor seg_cnt) {
  check_cuda_bf16(buf, "buf");
  TT_CHECK(buf.dim() == 2 && buf.is_contiguous() && buf.size(1) % 8 == 0, "ep_zero_pad: buf [rows, H]");
  TT_CHECK(seg_off.scalar_type() == torch::kInt32 && seg_cnt.scalar_type() == torch::kInt32 &&
               seg_off.numel() == seg_cnt.numel() + 1,
           "ep_zero_pad: seg_off int32 [E+1], seg_cnt int32 [E]");
  const int64_t E = seg_cnt.numel();
  if (E == 0) return;
  const c10::cuda::CUDAGuard guard(buf.device());
  dim3 grid(16, static_cast<unsigned>(E));
  ep::zero_pad_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<__nv_bfloat16*>(buf.data_ptr()),
                                                      seg_off.data_ptr<int>(), seg_cnt.data_ptr<int>(),
                                                      static_cast<int>(E), static_cast<int>(buf.size(1)),
                                                      buf.size(0));
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
