// Ulysses head<->sequence exchange for SEP attention, fused with its layout changes, on a
// symmetric heap (one NVLink domain).
//
// The reference (tinytron/model/modules/attn.py:226-268,367-373 with
// distributed/sequence_parallel/ulysses.py:7-26) expands the kv heads, permutes q/k/v into
// head-major tensors, runs an NCCL all-to-all per tensor and permutes back.  Here each
// direction is two kernels with no intermediate tensor:
//
//   pack      gathers this rank's outgoing chunks straight from the producer's layout
//             (the packed q|k|v projection output, or the attention output) into its
//             send slot [sp][B][T_loc][W] on the heap; for q|k|v it also applies the GQA
//             routing (rank c receives its q heads and only the kv heads they read, never
//             an expanded copy); the last block signals the peers.
//   exchange  waits for the peers, loads chunk `me` of every peer's slot over NVLink and
//             stores it straight into the consumer's layout: rows (b, c*T_loc + t) of the
//             full-sequence buffer the attention kernel reads, or the column block c of the
//             token-major output the c_proj GEMM reads.
//   exchange_qkv_grad (backward of the q|k|v direction) reads the peers' gradient chunks and
//             writes d(q|k|v) in the projection's layout, summing the contributions of the
//             ranks that share a kv head (fixed rank order: deterministic).
//
// Synchronisation uses the heap's device-side epoch (as the graph-safe all-reduce in
// comm.cu): pack reads epoch+1 and signals it; exchange waits for it, and its last block
// advances the epoch.  The two send slots alternate with the epoch's parity: a rank
// overwrites slot (e & 1) in call e + 2 only after its exchange of call e + 1 saw every
// peer's pack of e + 1, which each peer issued after finishing its exchange of call e.
// Every wait is bounded (kTimeoutPeer in the status word); nothing traps.
#include "runtime/comm_common.cuh"

namespace tt {
namespace comm {

constexpr int kUlThreads = 256;

struct UlPack {
  long long rs_b, rs_c, rs_t;  // source row of (b, c, t) = b*rs_b + c*rs_c + t*rs_t
  int ld_src;                  // source row stride (elements)
  int W;                       // chunk row width (elements, multiple of 8)
  int s1, s2;                  // segment boundaries inside a chunk row
  int base0[kMaxRanks], base1[kMaxRanks], base2[kMaxRanks];  // per-destination source columns
};

struct UlExch {
  long long ds_b, ds_c, ds_t;  // destination row of (b, c, t)
  int ld_out;                  // destination row stride (elements)
  int dcol_c;                  // destination column of chunk c = c * dcol_c
  int W;
};


// Each thread moves kUlUnroll 16-byte vectors per step, all loads issued before any store,
// so a thread keeps several NVLink (or HBM) round trips in flight instead of one; index
// math is 32-bit (the host checks that every vector count fits).
constexpr int kUlUnroll = 4;

__device__ __forceinline__ int ul_warp() { return static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5); }
__device__ __forceinline__ int ul_warps() { return static_cast<int>((gridDim.x * blockDim.x) >> 5); }

// Pack: one warp per row of the send slot; the row's coordinates (destination rank,
// batch, token) are decoded once and the lanes walk its 16-byte vectors (measured faster
// than decoding every vector).  The exchanges below keep one vector index per thread
// step: on NVLink that interleaving of many rows measured faster than a warp per row.
__global__ void __launch_bounds__(kUlThreads) ul_pack_kernel(PeerTable t, size_t slot_off, long long slot_bytes,
                                                            const __nv_bfloat16* __restrict__ src, int B, int T,
                                                            UlPack d) {
  const uint64_t e = dev_epoch_next(t);
  uint4* dst = reinterpret_cast<uint4*>(t.base[t.rank] + slot_off +
                                        static_cast<size_t>(e & 1ull) * static_cast<size_t>(slot_bytes));
  const int lane = threadIdx.x & 31;
  const int wv = d.W / 8;
  const int rows = t.world * B * T;  // (c, b, t)
  for (int row = ul_warp(); row < rows; row += ul_warps()) {
    const int tt = row % T;
    const int b = (row / T) % B;
    const int c = row / (T * B);
    const __nv_bfloat16* s = src + static_cast<size_t>(b * d.rs_b + c * d.rs_c + tt * d.rs_t) * d.ld_src;
    const int c0 = d.base0[c], c1 = d.base1[c] - d.s1, c2 = d.base2[c] - d.s2;
    uint4* o = dst + static_cast<size_t>(row) * wv;
    for (int v0 = lane; v0 < wv; v0 += 32 * kUlUnroll) {
      uint4 q[kUlUnroll];
#pragma unroll
      for (int u = 0; u < kUlUnroll; ++u) {
        const int v = v0 + 32 * u;
        if (v < wv) {
          const int w = v * 8;
          q[u] = *reinterpret_cast<const uint4*>(s + (w < d.s1 ? c0 : (w < d.s2 ? c1 : c2)) + w);
        }
      }
#pragma unroll
      for (int u = 0; u < kUlUnroll; ++u)
        if (v0 + 32 * u < wv) o[v0 + 32 * u] = q[u];
    }
  }
  grid_last_block(t, [&]() { signal_peers(t, e); });
}

__global__ void __launch_bounds__(kUlThreads) ul_exchange_kernel(PeerTable t, size_t slot_off, long long slot_bytes,
                                                                __nv_bfloat16* __restrict__ out, int B, int T,
                                                                UlExch d, int* status, uint64_t timeout_ns) {
  const uint64_t e = dev_epoch_next(t);
  if (block_wait_peers(t, e, status, timeout_ns)) {
    const size_t off = slot_off + static_cast<size_t>(e & 1ull) * static_cast<size_t>(slot_bytes);
    const int wv = d.W / 8;
    const int chunk_vecs = B * T * wv;
    const int total = chunk_vecs * t.world;
    const int stride = gridDim.x * blockDim.x;
    for (int i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += stride * kUlUnroll) {
      uint4 q[kUlUnroll];
#pragma unroll
      for (int u = 0; u < kUlUnroll; ++u) {  // chunk `me` of rank c, vector j
        const int i = i0 + u * stride;
        if (i < total) {
          const int c = i / chunk_vecs;
          const int j = i - c * chunk_vecs;
          q[u] = reinterpret_cast<const uint4*>(t.base[c] + off)[static_cast<long long>(t.rank) * chunk_vecs + j];
        }
      }
#pragma unroll
      for (int u = 0; u < kUlUnroll; ++u) {
        const int i = i0 + u * stride;
        if (i < total) {
          const int c = i / chunk_vecs;
          const int j = i - c * chunk_vecs;  // (b, t, v) inside the chunk
          const int vi = j % wv;
          const int row = j / wv;
          const int tt = row % T;
          const int b = row / T;
          const long long drow = b * d.ds_b + c * d.ds_c + tt * d.ds_t;
          *reinterpret_cast<uint4*>(out + static_cast<size_t>(drow) * d.ld_out + c * d.dcol_c + vi * 8) = q[u];
        }
      }
    }
  }
  grid_last_block(t, [&]() { *reinterpret_cast<volatile uint64_t*>(t.base[t.rank] + kDevEpochOff) = e; });
}

__global__ void __launch_bounds__(kUlThreads) ul_exchange_qkv_grad_kernel(
    PeerTable t, size_t slot_off, long long slot_bytes, __nv_bfloat16* __restrict__ dqkv, int B, int T, int Hq,
    int Hkv, int D, int hq_l, int hkv_l, UlPack kv, int* status, uint64_t timeout_ns) {
  const uint64_t e = dev_epoch_next(t);
  if (block_wait_peers(t, e, status, timeout_ns)) {
    const size_t off = slot_off + static_cast<size_t>(e & 1ull) * static_cast<size_t>(slot_bytes);
    const int W = (hq_l + 2 * hkv_l) * D;
    const int Wtot = (Hq + 2 * Hkv) * D;
    const int wv = Wtot / 8;
    const long long chunk_elems = static_cast<long long>(B) * T * W;
    const int total = B * T * wv;
    const int stride = gridDim.x * blockDim.x;
    auto src_of = [&](int c, int row, int w) {
      return reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(t.base[c] + off) +
                                            static_cast<long long>(t.rank) * chunk_elems +
                                            static_cast<long long>(row) * W + w);
    };
    auto add = [](float (&acc)[8], const uint4& q) {
      const uint32_t uw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(uw[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    };
    for (int i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += stride * kUlUnroll) {
      // q columns: one source each, loaded for all unrolled vectors before use; kv columns:
      // every rank whose kv range covers the head, summed in rank order (deterministic)
      uint4 qv[kUlUnroll];
#pragma unroll
      for (int u = 0; u < kUlUnroll; ++u) {
        const int i = i0 + u * stride;
        const int col = (i % wv) * 8;
        if (i < total && col < Hq * D) {
          const int h = col / D;
          qv[u] = *src_of(h / hq_l, i / wv, (h % hq_l) * D + col % D);
        }
      }
#pragma unroll
      for (int u = 0; u < kUlUnroll; ++u) {
        const int i = i0 + u * stride;
        if (i >= total) continue;
        const int row = i / wv;  // b * T + t
        const int col = (i % wv) * 8;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (col < Hq * D) {
          add(acc, qv[u]);
        } else {
          const bool is_v = col >= (Hq + Hkv) * D;
          const int kh = (col - (is_v ? (Hq + Hkv) * D : Hq * D)) / D;
          for (int c = 0; c < t.world; ++c) {
            const int k0 = kv.base1[c];
            if (kh >= k0 && kh < k0 + hkv_l) add(acc, *src_of(c, row, (hq_l + (is_v ? hkv_l : 0) + (kh - k0)) * D + col % D));
          }
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]);
        o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]);
        o.w = pack_bf16x2(acc[6], acc[7]);
        reinterpret_cast<uint4*>(dqkv)[i] = o;
      }
    }
  }
  grid_last_block(t, [&]() { *reinterpret_cast<volatile uint64_t*>(t.base[t.rank] + kDevEpochOff) = e; });
}

// Pack grid: one warp per row (8 rows per 256-thread CTA), up to eight CTAs per SM (the
// kernel keeps no per-block scratch, only the heap's last-block counter).
static int ul_pack_grid(int device, long long rows) {
  const long long blocks = (rows + kUlThreads / 32 - 1) / (kUlThreads / 32);
  return static_cast<int>(std::max<long long>(1, std::min<long long>(blocks, 8ll * num_sms(device))));
}

static int ul_grid(int device, long long vecs) {
  TT_CHECK(vecs < (1ll << 31), "ulysses: exchange larger than 2^31 16-byte vectors");
  const long long per_thread = (vecs + kUlUnroll - 1) / kUlUnroll;
  return std::max(1, std::min(grid_blocks(device, per_thread, kUlThreads), 4 * num_sms(device)));
}

// Host bounds of the row maps: every (b, c, t) row of a pack source or an exchange
// destination lies inside `t`'s rows, and the column ranges inside its row width.
static void ul_check_rows(const torch::Tensor& t, int64_t B, int64_t T, int world, const std::vector<int64_t>& rows,
                          const char* what) {
  TT_CHECK(B >= 0 && T >= 0 && rows[0] >= 0 && rows[1] >= 0 && rows[2] >= 0,
           std::string("ulysses: negative size or row stride in ") + what);
  const int64_t ld = t.size(-1);
  const int64_t n_rows = ld > 0 ? t.numel() / ld : 0;
  if (B > 0 && T > 0)
    TT_CHECK((B - 1) * rows[0] + static_cast<int64_t>(world - 1) * rows[1] + (T - 1) * rows[2] < n_rows,
             std::string("ulysses: row map past the last row of ") + what);
}

static void ul_check_slots(int64_t gid, int64_t slot_offset, int64_t slot_bytes, long long need) {
  TT_CHECK(slot_offset % 256 == 0 && slot_bytes % 256 == 0 && need <= slot_bytes &&
               slot_offset + 2 * slot_bytes <= static_cast<int64_t>(group_bytes(gid)),
           "ulysses: send slots outside the heap or too small");
}

static UlPack make_pack(std::vector<int64_t> rows, int64_t ld_src, int64_t W, int64_t s1, int64_t s2,
                        std::vector<int64_t> b0, std::vector<int64_t> b1, std::vector<int64_t> b2, int world) {
  TT_CHECK(rows.size() == 3 && static_cast<int>(b0.size()) == world && static_cast<int>(b1.size()) == world &&
               static_cast<int>(b2.size()) == world, "ulysses: bad pack descriptor");
  TT_CHECK(W % 8 == 0 && s1 % 8 == 0 && s2 % 8 == 0 && ld_src % 8 == 0, "ulysses: widths must be multiples of 8");
  UlPack d{};
  d.rs_b = rows[0];
  d.rs_c = rows[1];
  d.rs_t = rows[2];
  d.ld_src = static_cast<int>(ld_src);
  d.W = static_cast<int>(W);
  d.s1 = static_cast<int>(s1);
  d.s2 = static_cast<int>(s2);
  for (int c = 0; c < world; ++c) {
    TT_CHECK(b0[c] % 8 == 0 && b1[c] % 8 == 0 && b2[c] % 8 == 0, "ulysses: column bases must be multiples of 8");
    d.base0[c] = static_cast<int>(b0[c]);
    d.base1[c] = static_cast<int>(b1[c]);
    d.base2[c] = static_cast<int>(b2[c]);
  }
  return d;
}

// Pack this rank's outgoing chunks [sp][B][T][W] into send slot (epoch + 1) and signal.
void ul_pack(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor src, int64_t B, int64_t T,
             std::vector<int64_t> rows, int64_t W, int64_t s1, int64_t s2, std::vector<int64_t> b0,
             std::vector<int64_t> b1, std::vector<int64_t> b2) {
  check_cuda_bf16(src, "src");
  TT_CHECK(src.is_contiguous() && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "ulysses: src layout");
  const PeerTable t = group_table(gid);
  TT_CHECK(src.get_device() == group_device(gid), "ulysses: src is not on the heap's device");
  const UlPack d = make_pack(rows, src.size(-1), W, s1, s2, b0, b1, b2, t.world);
  ul_check_rows(src, B, T, t.world, rows, "src");
  const int64_t ld = src.size(-1);
  TT_CHECK(0 <= s1 && s1 <= s2 && s2 <= W, "ulysses: segments must satisfy 0 <= s1 <= s2 <= W");
  for (int c = 0; c < t.world; ++c)  // the three column segments of destination c inside a source row
    TT_CHECK(b0[c] >= 0 && b0[c] + s1 <= ld && b1[c] >= 0 && b1[c] + (s2 - s1) <= ld && b2[c] >= 0 &&
                 b2[c] + (W - s2) <= ld,
             "ulysses: pack columns outside the source row");
  const long long vecs = static_cast<long long>(t.world) * B * T * (W / 8);
  ul_check_slots(gid, slot_offset, slot_bytes, vecs * 16);
  const int device = group_device(gid);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  TT_CHECK(vecs < (1ll << 31), "ulysses: exchange larger than 2^31 16-byte vectors");
  ul_pack_kernel<<<ul_pack_grid(device, static_cast<long long>(t.world) * B * T), kUlThreads, 0, cur_stream()>>>(
      t, static_cast<size_t>(slot_offset), slot_bytes, reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()),
      static_cast<int>(B), static_cast<int>(T), d);
  TT_CUDA_CHECK(cudaGetLastError());
}

// Wait for the peers' packs, store chunk `me` of every peer into `out` (row / column remap).
void ul_exchange(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor out, int64_t B, int64_t T,
                 std::vector<int64_t> rows, int64_t dcol_c, int64_t W) {
  check_cuda_bf16(out, "out");
  TT_CHECK(out.is_contiguous() && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0 && out.size(-1) % 8 == 0 &&
               W % 8 == 0 && dcol_c % 8 == 0 && rows.size() == 3, "ulysses: out layout");
  const PeerTable t = group_table(gid);
  TT_CHECK(out.get_device() == group_device(gid), "ulysses: out is not on the heap's device");
  ul_check_rows(out, B, T, t.world, rows, "out");
  TT_CHECK(dcol_c >= 0 && static_cast<int64_t>(t.world - 1) * dcol_c + W <= out.size(-1),
           "ulysses: exchange columns outside the destination row");
  UlExch d{};
  d.ds_b = rows[0];
  d.ds_c = rows[1];
  d.ds_t = rows[2];
  d.ld_out = static_cast<int>(out.size(-1));
  d.dcol_c = static_cast<int>(dcol_c);
  d.W = static_cast<int>(W);
  const long long vecs = static_cast<long long>(t.world) * B * T * (W / 8);
  ul_check_slots(gid, slot_offset, slot_bytes, vecs * 16);
  const int device = group_device(gid);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  ul_exchange_kernel<<<ul_grid(device, vecs), kUlThreads, 0, cur_stream()>>>(
      t, static_cast<size_t>(slot_offset), slot_bytes, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      static_cast<int>(B), static_cast<int>(T), d, device_status_ptr(device), wait_timeout_ns());
  TT_CUDA_CHECK(cudaGetLastError());
}

// Backward of the q|k|v direction: d(q|k|v) of this rank's tokens from the peers' chunks.
void ul_exchange_qkv_grad(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor dqkv, int64_t B,
                          int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int64_t hq_l, int64_t hkv_l,
                          std::vector<int64_t> kv0) {
  check_cuda_bf16(dqkv, "dqkv");
  const PeerTable t = group_table(gid);
  TT_CHECK(dqkv.is_contiguous() && dqkv.numel() == B * T * (Hq + 2 * Hkv) * D && D % 8 == 0 &&
               static_cast<int>(kv0.size()) == t.world, "ulysses: dqkv layout");
  TT_CHECK(dqkv.get_device() == group_device(gid), "ulysses: dqkv is not on the heap's device");
  TT_CHECK(hq_l >= 1 && hq_l * t.world == Hq && hkv_l >= 1 && hkv_l <= Hkv,
           "ulysses: q heads split evenly over the ranks, 1 <= kv heads per rank <= Hkv");
  UlPack kv{};
  for (int c = 0; c < t.world; ++c) {
    TT_CHECK(kv0[c] >= 0 && kv0[c] + hkv_l <= Hkv, "ulysses: a rank's kv heads outside [0, Hkv)");
    kv.base1[c] = static_cast<int>(kv0[c]);
  }
  const long long W = (hq_l + 2 * hkv_l) * D;
  ul_check_slots(gid, slot_offset, slot_bytes, static_cast<long long>(t.world) * B * T * W * 2);
  const long long vecs = B * T * (Hq + 2 * Hkv) * D / 8;
  const int device = group_device(gid);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  ul_exchange_qkv_grad_kernel<<<ul_grid(device, vecs), kUlThreads, 0, cur_stream()>>>(
      t, static_cast<size_t>(slot_offset), slot_bytes, reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
      static_cast<int>(B), static_cast<int>(T), static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(D),
      static_cast<int>(hq_l), static_cast<int>(hkv_l), kv, device_status_ptr(device), wait_timeout_ns());
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace comm
}  // namespace tt
