// tt_comm: symmetric-memory communication runtime for one process per GPU over
// NVLink 5 / NVSwitch, plus the collectives that run on it as device-initiated
// peer loads and stores from inside ordinary kernels.
//
// A group owns one device buffer ("heap") per rank, allocated with cudaMalloc and
// mapped into every other rank's address space through CUDA IPC handles (the
// Python layer exchanges the 64-byte handles over the process group).  Kernels get
// the table of peer base pointers by value and load from / store to the peers'
// heaps directly: plain NVLink loads and stores, no TMA, no multicast.
//
// Heap layout (byte offsets from each heap's base, identical on every rank):
//   [0, 64)              flags[8]     uint64, flags[s] is written only by rank s
//   [1024, 3072)         pads[8][64]  fp32,   pads[s][*] is written only by rank s
//   [4096, 4104)         grid arrival counter (local use only)
//   [8192, 16384)        per-block partial sums (local use only)
//   [65536, bytes)       user region (tensors laid out by the Python allocator)
//
// Synchronisation.  Every rank of a group issues the same collectives in the same
// order, so a host-side epoch counter per group advances identically everywhere.
// A kernel "signals" epoch e by storing e into flags[my_rank] of every peer with
// st.release.sys after a system-scope fence; it "waits" for e by spinning with
// ld.acquire.sys on its own flags[p] until flags[p] >= e for every peer p.  Every
// wait is bounded by %globaltimer: on expiry it records kTimeoutPeer in the device
// status word and the kernel returns early (its outputs are then invalid; the
// host raises from tinytron_b200.ops.check_status).  Nothing here traps.
//
// Collectives (the reference runs these as NCCL calls: trainer.py DDP all-reduce,
// distributed/zero1/distributed_optimizer.py:106-119 per-tensor broadcasts,
// model/modules/attn.py:364 and mlp.py:221 inference all-reduces):
//   * barrier                           all ranks reach the same epoch
//   * all_reduce (one-shot)             out = sum_p peer_p[in] (+ residual), bf16/fp32
//   * reduce_scatter_sumsq  (ZeRO-1)    grad[lo:hi] = scale * sum_p peer_p.grad[lo:hi],
//                                       plus this rank's sum of squares published to
//                                       every peer's pad (for the global clip norm)
//   * adamw_allgather       (ZeRO-1)    clip coefficient from the peers' pads, AdamW on
//                                       the owned shard, fp32 master shard stored into
//                                       every peer's parameter buffer
//   * shadow_refresh                    waits for the all-gather, rewrites the bf16
//                                       shadow of the shards other ranks updated
//   * all_to_all (equal split)          out[c] = rank c's chunk for this rank, by peer
//                                       loads (Ulysses head<->sequence exchange)
#include "runtime/comm_common.cuh"

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace tt {
namespace comm {

// ------------------------------------------------------------------ kernels
__global__ void barrier_kernel(PeerTable t, uint64_t e, int* status, uint64_t timeout_ns, int do_signal) {
  if (threadIdx.x != 0) return;
  if (do_signal) signal_peers(t, e);
  wait_peers(t, e, status, timeout_ns);
}

// One-shot all-reduce over the group: out[i] = sum_p peer_p[in_off][i] (+ residual[i]).
// Every rank sums in the same rank order, so all ranks get bit-identical results.
template <typename T>
__global__ void allreduce_kernel(PeerTable t, size_t in_off, T* __restrict__ out, const T* __restrict__ residual,
                                 long long n, uint64_t e, int* status, uint64_t timeout_ns) {
  if (blockIdx.x == 0 && threadIdx.x == 0) signal_peers(t, e);  // our slot is complete (stream order)
  if (!block_wait_peers(t, e, status, timeout_ns)) return;
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  const long long nv = n / V;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float acc[V];
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = 0.f;
    for (int p = 0; p < t.world; ++p) {
      const uint4 q = reinterpret_cast<const uint4*>(t.base[p] + in_off)[i];
      const T* qv = reinterpret_cast<const T*>(&q);
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] += static_cast<float>(qv[k]);
    }
    if (residual != nullptr) {
      const uint4 r = reinterpret_cast<const uint4*>(residual)[i];
      const T* rv = reinterpret_cast<const T*>(&r);
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] += static_cast<float>(rv[k]);
    }
    uint4 o;
    T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < V; ++k) ov[k] = static_cast<T>(acc[k]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
  for (long long i = nv * V + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float acc = 0.f;
    for (int p = 0; p < t.world; ++p) acc += static_cast<float>(reinterpret_cast<const T*>(t.base[p] + in_off)[i]);
    if (residual != nullptr) acc += static_cast<float>(residual[i]);
    out[i] = static_cast<T>(acc);
  }
}

// Equal-split all-to-all by peer loads: out[c] = peer_c.slot[my_rank] for every rank c
// (chunk = chunk_bytes, a multiple of 16).  Each rank's slot holds its `world` outgoing
// chunks; the start barrier makes every slot complete before anyone reads.
__global__ void alltoall_kernel(PeerTable t, size_t slot_off, long long chunk_bytes, char* __restrict__ out,
                                uint64_t e, int* status, uint64_t timeout_ns) {
  if (blockIdx.x == 0 && threadIdx.x == 0) signal_peers(t, e);
  if (!block_wait_peers(t, e, status, timeout_ns)) return;
  const long long nv = chunk_bytes / 16;
  const long long total = nv * t.world;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int c = static_cast<int>(i / nv);
    const long long v = i - c * nv;
    const uint4* src = reinterpret_cast<const uint4*>(t.base[c] + slot_off + t.rank * chunk_bytes);
    reinterpret_cast<uint4*>(out + c * chunk_bytes)[v] = src[v];
  }
}

// ZeRO-1 gradient reduce-scatter.  grad[lo:hi] (this rank's shard, in place in its
// own heap) = scale * sum_p peer_p.grad[lo:hi].  Also the sums of squares of the
// reduced shard split at `split` (elements < split: dense parameters; >= split:
// expert parameters), reduced deterministically over blocks and stored into
// pads[my_rank][0..1] of every peer before signalling epoch e_done.
// sq_local != nullptr (bucketed reduce-scatter, overlapped with the backward): the block
// sums go to sq_local[0..1] on this rank only, and no completion epoch is signalled;
// publish_sumsq_kernel later publishes the total over all buckets.
__global__ void rs_sumsq_kernel(PeerTable t, size_t grad_off, long long lo, long long hi, long long split,
                                float scale, uint64_t e_start, uint64_t e_done, int* status, uint64_t timeout_ns,
                                float* sq_local) {
  if (blockIdx.x == 0 && threadIdx.x == 0) signal_peers(t, e_start);  // our grads are final (stream order)
  if (!block_wait_peers(t, e_start, status, timeout_ns)) return;
  float sd = 0.f, se = 0.f;
  const long long n4 = (hi - lo) / 4;  // lo, hi are multiples of 4 (checked on the host)
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  float* mine = reinterpret_cast<float*>(t.base[t.rank] + grad_off) + lo;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < t.world; ++p) {
      const float4 g = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(t.base[p] + grad_off) + lo)[i];
      acc.x += g.x;
      acc.y += g.y;
      acc.z += g.z;
      acc.w += g.w;
    }
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
    reinterpret_cast<float4*>(mine)[i] = acc;
    const float s = acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
    if (lo + 4 * i < split) sd += s;  // split is a multiple of 4 (alignment of the flat layout)
    else se += s;
  }
  const float2 bs = block_sum2(sd, se);
  float* partial = reinterpret_cast<float*>(t.base[t.rank] + kPartialOff);
  if (threadIdx.x == 0) {
    partial[2 * blockIdx.x] = bs.x;
    partial[2 * blockIdx.x + 1] = bs.y;
  }
  grid_last_block(t, [&]() {
    float d = 0.f, x = 0.f;
    for (unsigned int b = 0; b < gridDim.x; ++b) {  // fixed order: deterministic
      d += partial[2 * b];
      x += partial[2 * b + 1];
    }
    if (sq_local != nullptr) {
      sq_local[0] = d;
      sq_local[1] = x;
      return;
    }
    for (int p = 0; p < t.world; ++p) {
      float* pad = pad_ptr(t, p, t.rank);
      pad[0] = d;
      pad[1] = x;
    }
    signal_peers(t, e_done);
  });
}

// One thread: total the per-bucket sums of squares (fixed order), publish them into every
// peer's pad and signal epoch e.
__global__ void publish_sumsq_kernel(PeerTable t, const float* __restrict__ sq, int n_buckets, uint64_t e) {
  if (threadIdx.x != 0) return;
  float d = 0.f, x = 0.f;
  for (int b = 0; b < n_buckets; ++b) {
    d += sq[2 * b];
    x += sq[2 * b + 1];
  }
  for (int p = 0; p < t.world; ++p) {
    float* pad = pad_ptr(t, p, t.rank);
    pad[0] = d;
    pad[1] = x;
  }
  signal_peers(t, e);
}

struct AdamArgs {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, max_norm;
};

// ZeRO-1 update + all-gather.  Waits for every peer's partial sums of squares
// (epoch e_pads), forms the global norm and clip coefficient (same order on every
// rank), applies AdamW to this rank's shard and stores the new fp32 master shard
// into every peer's parameter buffer; the bf16 shadow of the owned shard is
// written locally.  The last block signals e_done.
__global__ void adamw_allgather_kernel(PeerTable t, size_t data_off, size_t grad_off, __nv_bfloat16* __restrict__ p16,
                                       float* __restrict__ m, float* __restrict__ v, long long lo, long long hi,
                                       AdamArgs a, const float* __restrict__ extra_sq, float* __restrict__ norm_out,
                                       uint64_t e_pads, uint64_t e_done, int* status, uint64_t timeout_ns) {
  if (!block_wait_peers(t, e_pads, status, timeout_ns)) return;
  __shared__ float coef_s;
  if (threadIdx.x == 0) {
    float sq = 0.f;
    for (int p = 0; p < t.world; ++p) {
      const float* pad = pad_ptr(t, t.rank, p);
      sq += pad[0] + pad[1];
    }
    if (extra_sq != nullptr) sq += *extra_sq;
    const float nrm = sqrtf(sq);
    coef_s = a.max_norm > 0.f ? fminf(a.max_norm / (nrm + 1e-6f), 1.0f) : 1.0f;
    if (blockIdx.x == 0 && norm_out != nullptr) {
      norm_out[0] = nrm;
      norm_out[1] = coef_s;
    }
  }
  __syncthreads();
  const float gs = coef_s;
  const float step = a.lr / a.bc1;
  const float decay = 1.0f - a.lr * a.wd;
  const long long n4 = (hi - lo) / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  float* pl = reinterpret_cast<float*>(t.base[t.rank] + data_off) + lo;
  const float* gl = reinterpret_cast<const float*>(t.base[t.rank] + grad_off) + lo;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pv = reinterpret_cast<float4*>(pl)[i];
    const float4 gv = reinterpret_cast<const float4*>(gl)[i];
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = &pv.x;
    const float* gp = &gv.x;
    float* mp = &mv.x;
    float* vp = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gr = gp[k] * gs;
      pp[k] *= decay;
      mp[k] = mp[k] + (1.0f - a.beta1) * (gr - mp[k]);
      vp[k] = a.beta2 * vp[k] + (1.0f - a.beta2) * gr * gr;
      const float denom = sqrtf(vp[k]) / a.bc2_sqrt + a.eps;
      pp[k] -= step * (mp[k] / denom);
    }
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
    for (int p = 0; p < t.world; ++p)  // own heap included: one code path for every destination
      reinterpret_cast<float4*>(reinterpret_cast<float*>(t.base[p] + data_off) + lo)[i] = pv;
    if (p16 != nullptr) {
      uint2 o;
      o.x = pack_bf16x2(pv.x, pv.y);
      o.y = pack_bf16x2(pv.z, pv.w);
      reinterpret_cast<uint2*>(p16 + lo)[i] = o;
    }
  }
  grid_last_block(t, [&]() { signal_peers(t, e_done); });
}

// Waits for the all-gather epoch, then rewrites the bf16 shadow of [0, lo) and
// [hi, n) from the fp32 masters the peers stored.
__global__ void shadow_refresh_kernel(PeerTable t, size_t data_off, __nv_bfloat16* __restrict__ p16, long long lo,
                                      long long hi, long long n, uint64_t e, int* status, uint64_t timeout_ns) {
  if (!block_wait_peers(t, e, status, timeout_ns)) return;
  if (p16 == nullptr) return;
  const float* d = reinterpret_cast<const float*>(t.base[t.rank] + data_off);
  const long long n4 = n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const long long e0 = 4 * i;
    if (e0 >= lo && e0 < hi) continue;
    const float4 pv = reinterpret_cast<const float4*>(d)[i];
    uint2 o;
    o.x = pack_bf16x2(pv.x, pv.y);
    o.y = pack_bf16x2(pv.z, pv.w);
    reinterpret_cast<uint2*>(p16)[i] = o;
  }
}

// ------------------------------------------------------------------ replayable all-reduce
// Graph-capturable all-reduce / broadcast (SEP inference: row-parallel partial sums, and
// the decode step is one CUDA graph).  Two kernels per call:
//   publish:  e = dev_epoch + 1; copy `in` into this rank's slot (e & 1); the last block
//             signals e to every peer.
//   reduce:   e = dev_epoch + 1; wait for every peer's e; out = sum over ranks (or the
//             root's slot only) in rank order (+ residual); the last block stores
//             dev_epoch = e.
// Slots alternate with the epoch's parity: a rank rewrites slot (e & 1) at call e + 2 only
// after its reduce of call e + 1 saw every peer's publish of e + 1, which each peer issued
// after finishing its reduce of call e (stream order), i.e. after reading that slot.

__global__ void replay_publish_kernel(PeerTable t, size_t slot_off, long long slot_bytes, const char* __restrict__ in,
                                      long long bytes) {
  const uint64_t e = dev_epoch_next(t);
  char* dst = t.base[t.rank] + slot_off + static_cast<size_t>(e & 1ull) * static_cast<size_t>(slot_bytes);
  const long long nv = bytes / 16;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(in)[i];
  grid_last_block(t, [&]() { signal_peers(t, e); });
}

template <typename T>
__global__ void replay_reduce_kernel(PeerTable t, size_t slot_off, long long slot_bytes, T* __restrict__ out,
                                     const T* __restrict__ residual, long long n, int root, int* status,
                                     uint64_t timeout_ns) {
  const uint64_t e = dev_epoch_next(t);
  const size_t off = slot_off + static_cast<size_t>(e & 1ull) * static_cast<size_t>(slot_bytes);
  bool ok = block_wait_peers(t, e, status, timeout_ns);
  if (ok) {
    constexpr int V = 16 / sizeof(T);
    const long long nv = n / V;
    const int p0 = root >= 0 ? root : 0, p1 = root >= 0 ? root + 1 : t.world;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
      float acc[V];
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] = 0.f;
      for (int p = p0; p < p1; ++p) {
        const uint4 q = reinterpret_cast<const uint4*>(t.base[p] + off)[i];
        const T* qv = reinterpret_cast<const T*>(&q);
#pragma unroll
        for (int k = 0; k < V; ++k) acc[k] += static_cast<float>(qv[k]);
      }
      if (residual != nullptr) {
        const uint4 r = reinterpret_cast<const uint4*>(residual)[i];
        const T* rv = reinterpret_cast<const T*>(&r);
#pragma unroll
        for (int k = 0; k < V; ++k) acc[k] += static_cast<float>(rv[k]);
      }
      uint4 o;
      T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int k = 0; k < V; ++k) ov[k] = static_cast<T>(acc[k]);
      reinterpret_cast<uint4*>(out)[i] = o;
    }
  }
  // Advance the epoch even after a timeout (the status word is set and the host raises),
  // so every rank's epoch keeps counting calls.
  grid_last_block(t, [&]() { *reinterpret_cast<volatile uint64_t*>(t.base[t.rank] + kDevEpochOff) = e; });
}

// ------------------------------------------------------------------ host side
struct Group {
  int device = -1;
  int rank = 0;
  int world = 1;
  size_t bytes = 0;
  char* heap = nullptr;
  char* peer[kMaxRanks] = {nullptr};
  bool opened[kMaxRanks] = {false};
  bool emulated = false;  // peers are other groups of this process (single-GPU test mode)
  uint64_t epoch = 0;
};

static std::mutex g_mu;
static std::vector<Group*> g_groups;

static Group& get(int64_t gid) {
  std::lock_guard<std::mutex> lock(g_mu);
  TT_CHECK(gid >= 0 && gid < static_cast<int64_t>(g_groups.size()) && g_groups[gid] != nullptr,
           "comm: invalid group id");
  return *g_groups[gid];
}

static PeerTable table(const Group& g) {
  PeerTable t;
  for (int i = 0; i < kMaxRanks; ++i) t.base[i] = g.peer[i];
  t.rank = g.rank;
  t.world = g.world;
  for (int i = 0; i < g.world; ++i) TT_CHECK(g.peer[i] != nullptr, "comm: peers not opened");
  return t;
}

// Bound on every device-side wait of a collective: TT_COMM_TIMEOUT_S (default 60 s;
// far above any legitimate skew between ranks), changeable with comm_set_timeout.
static std::atomic<uint64_t> g_timeout_ns{0};
static uint64_t timeout_ns() {
  uint64_t ns = g_timeout_ns.load();
  if (ns == 0) {
    const char* s = std::getenv("TT_COMM_TIMEOUT_S");
    const double sec = s ? std::atof(s) : 60.0;
    ns = static_cast<uint64_t>((sec > 0 ? sec : 60.0) * 1e9);
    g_timeout_ns.store(ns);
  }
  return ns;
}

void comm_set_timeout(double seconds) {
  TT_CHECK(seconds > 0, "comm: timeout must be positive");
  g_timeout_ns.store(static_cast<uint64_t>(seconds * 1e9));
}

static int grid_for(int device, long long work_items, int threads) {
  const int dev_sms = num_sms(device);
  long long blocks = (work_items + threads - 1) / threads;
  blocks = std::max<long long>(1, std::min<long long>(blocks, std::min(2 * dev_sms, kMaxBlocks)));
  return static_cast<int>(blocks);
}

int64_t comm_create(int64_t device, int64_t bytes) {
  TT_CHECK(bytes > static_cast<int64_t>(kUserOff), "comm: heap too small");
  auto* g = new Group();
  g->device = static_cast<int>(device);
  g->bytes = static_cast<size_t>(bytes);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  TT_CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&g->heap), g->bytes));
  TT_CUDA_CHECK(cudaMemset(g->heap, 0, kUserOff));
  TT_CUDA_CHECK(cudaDeviceSynchronize());
  std::lock_guard<std::mutex> lock(g_mu);
  g_groups.push_back(g);
  return static_cast<int64_t>(g_groups.size() - 1);
}

torch::Tensor comm_ipc_handle(int64_t gid) {
  Group& g = get(gid);
  cudaIpcMemHandle_t h;
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  TT_CUDA_CHECK(cudaIpcGetMemHandle(&h, g.heap));
  auto out = torch::empty({static_cast<int64_t>(sizeof(h))}, torch::kUInt8);
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

// handles: uint8 [world, 64] (row r = rank r's heap handle; our own row is ignored).
void comm_open(int64_t gid, int64_t rank, int64_t world, torch::Tensor handles) {
  Group& g = get(gid);
  TT_CHECK(world >= 1 && world <= kMaxRanks, "comm: world size must be 1..8");
  TT_CHECK(rank >= 0 && rank < world, "comm: bad rank");
  TT_CHECK(handles.dtype() == torch::kUInt8 && handles.dim() == 2 && handles.size(0) == world &&
               handles.size(1) == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)),
           "comm: handles must be uint8 [world, 64]");
  auto h = handles.contiguous().cpu();
  g.rank = static_cast<int>(rank);
  g.world = static_cast<int>(world);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  for (int p = 0; p < g.world; ++p) {
    if (p == g.rank) {
      g.peer[p] = g.heap;
      continue;
    }
    cudaIpcMemHandle_t mh;
    std::memcpy(&mh, h.data_ptr<uint8_t>() + p * sizeof(mh), sizeof(mh));
    void* ptr = nullptr;
    TT_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, mh, cudaIpcMemLazyEnablePeerAccess));
    g.peer[p] = static_cast<char*>(ptr);
    g.opened[p] = true;
  }
}

// Single-GPU test mode: groups gids[0..W-1] of this process act as the W ranks of
// one group (peer pointers are the other groups' heaps, all on one device).  The
// collectives are then launched rank by rank with waits disabled (the launch order
// supplies the ordering the epochs would), so no kernel ever waits on another.
//
// With waits=true the groups keep their real (bounded) waits: used only by the
// test that launches ONE rank's barrier whose peer never signals, to check that
// the wait gives up, records kTimeoutPeer and returns.
void comm_open_emulated(std::vector<int64_t> gids, bool waits) {
  const int w = static_cast<int>(gids.size());
  TT_CHECK(w >= 1 && w <= kMaxRanks, "comm: emulated world size must be 1..8");
  for (int r = 0; r < w; ++r) {
    Group& g = get(gids[r]);
    g.rank = r;
    g.world = w;
    g.emulated = !waits;
    for (int p = 0; p < w; ++p) g.peer[p] = get(gids[p]).heap;
  }
}

torch::Tensor comm_view(int64_t gid, int64_t offset_bytes, std::vector<int64_t> shape, int64_t dtype_code) {
  Group& g = get(gid);
  const auto dt = static_cast<c10::ScalarType>(dtype_code);
  int64_t numel = 1;
  for (auto s : shape) numel *= s;
  const int64_t nbytes = numel * static_cast<int64_t>(c10::elementSize(dt));
  TT_CHECK(offset_bytes >= static_cast<int64_t>(kUserOff) && offset_bytes % 256 == 0, "comm: bad view offset");
  TT_CHECK(offset_bytes + nbytes <= static_cast<int64_t>(g.bytes), "comm: view exceeds the heap");
  auto opts = torch::TensorOptions().dtype(dt).device(torch::kCUDA, g.device);
  return torch::from_blob(g.heap + offset_bytes, shape, opts);
}

int64_t comm_user_offset() { return static_cast<int64_t>(kUserOff); }

int64_t comm_heap_base(int64_t gid) { return static_cast<int64_t>(reinterpret_cast<uintptr_t>(get(gid).heap)); }

static uint64_t next_epoch(Group& g) { return ++g.epoch; }

// signal == false leaves this rank's flag unset (host-side fault injection: the
// peers' bounded waits then expire and record kTimeoutPeer).
void comm_barrier(int64_t gid, bool signal) {
  Group& g = get(gid);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  if (g.emulated) return;
  const uint64_t e = next_epoch(g);
  barrier_kernel<<<1, 32, 0, cur_stream()>>>(table(g), e, device_status_ptr(g.device), timeout_ns(), signal ? 1 : 0);
  TT_CUDA_CHECK(cudaGetLastError());
}

// out = sum over ranks of the heap region [in_offset, +numel) (+ residual).
void comm_all_reduce(int64_t gid, int64_t in_offset, torch::Tensor out, c10::optional<torch::Tensor> residual) {
  Group& g = get(gid);
  TT_CHECK(out.is_cuda() && out.is_contiguous(), "comm_all_reduce: out must be contiguous CUDA");
  TT_CHECK(out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32,
           "comm_all_reduce: bf16 or fp32");
  const long long n = out.numel();
  TT_CHECK(in_offset % 16 == 0 && in_offset >= static_cast<int64_t>(kUserOff) &&
               in_offset + n * static_cast<long long>(out.element_size()) <= static_cast<int64_t>(g.bytes),
           "comm_all_reduce: input region outside the heap");
  TT_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "comm_all_reduce: out must be 16-byte aligned");
  const void* res = nullptr;
  if (residual.has_value()) {
    TT_CHECK(residual->scalar_type() == out.scalar_type() && residual->numel() == n && residual->is_contiguous() &&
                 reinterpret_cast<uintptr_t>(residual->data_ptr()) % 16 == 0,
             "comm_all_reduce: residual must match out");
    res = residual->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  // Emulated mode waits for epoch 0 (always satisfied): the launch order of the
  // emulated ranks already makes every input complete.
  const uint64_t e = g.emulated ? 0ull : next_epoch(g);
  const int threads = 256;
  const int grid = grid_for(g.device, std::max<long long>(1, n / 8), threads);
  const PeerTable t = table(g);
  int* st = device_status_ptr(g.device);
  if (out.scalar_type() == torch::kBFloat16) {
    allreduce_kernel<__nv_bfloat16><<<grid, threads, 0, cur_stream()>>>(
        t, static_cast<size_t>(in_offset), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(res), n, e, st, timeout_ns());
  } else {
    allreduce_kernel<float><<<grid, threads, 0, cur_stream()>>>(
        t, static_cast<size_t>(in_offset), out.data_ptr<float>(), reinterpret_cast<const float*>(res), n, e, st,
        timeout_ns());
  }
  TT_CUDA_CHECK(cudaGetLastError());
}

// out (contiguous, world * chunk_bytes) <- chunk my_rank of every rank's slot at slot_offset.
void comm_all_to_all(int64_t gid, int64_t slot_offset, torch::Tensor out) {
  Group& g = get(gid);
  TT_CHECK(out.is_cuda() && out.is_contiguous(), "comm_all_to_all: out must be contiguous CUDA");
  const long long bytes = out.numel() * static_cast<long long>(out.element_size());
  TT_CHECK(bytes % (16LL * g.world) == 0, "comm_all_to_all: chunk size must be a multiple of 16 bytes");
  TT_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "comm_all_to_all: out must be 16-byte aligned");
  TT_CHECK(slot_offset % 256 == 0 && slot_offset >= static_cast<int64_t>(kUserOff) &&
               slot_offset + bytes <= static_cast<int64_t>(g.bytes),
           "comm_all_to_all: slot outside the heap");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  const uint64_t e = g.emulated ? 0ull : next_epoch(g);
  const int threads = 256;
  const int grid = grid_for(g.device, std::max<long long>(1, bytes / 16), threads);
  alltoall_kernel<<<grid, threads, 0, cur_stream()>>>(table(g), static_cast<size_t>(slot_offset), bytes / g.world,
                                                      static_cast<char*>(out.data_ptr()), e,
                                                      device_status_ptr(g.device), timeout_ns());
  TT_CUDA_CHECK(cudaGetLastError());
}

// ZeRO-1: reduce-scatter the fp32 gradient buffer at grad_offset (numel elements,
// identical layout on every rank) into this rank's [lo, hi) in place.
void comm_reduce_scatter_sumsq(int64_t gid, int64_t grad_offset, int64_t lo, int64_t hi, int64_t split,
                               double scale) {
  Group& g = get(gid);
  TT_CHECK(lo % 4 == 0 && hi % 4 == 0 && split % 4 == 0 && lo <= hi, "comm_rs: lo/hi/split must be multiples of 4");
  TT_CHECK(grad_offset % 256 == 0 && grad_offset + hi * 4 <= static_cast<int64_t>(g.bytes), "comm_rs: bad region");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  const uint64_t e0 = next_epoch(g), e1 = next_epoch(g);
  const int threads = 512;
  const int grid = grid_for(g.device, std::max<long long>(1, (hi - lo) / 4), threads);
  rs_sumsq_kernel<<<grid, threads, 0, cur_stream()>>>(table(g), static_cast<size_t>(grad_offset), lo, hi, split,
                                                       static_cast<float>(scale), g.emulated ? 0ull : e0,
                                                       g.emulated ? 0ull : e1, device_status_ptr(g.device),
                                                       timeout_ns(), nullptr);
  TT_CUDA_CHECK(cudaGetLastError());
}

// One bucket of a reduce-scatter that overlaps the backward: grad[lo:hi] = scale * sum over
// ranks (in place), its sums of squares into sq_local (fp32 [2], this rank's memory).  The
// grid is capped at max_blocks so the kernel shares the GPU with the backward's GEMMs.
void comm_reduce_scatter_bucket(int64_t gid, int64_t grad_offset, int64_t lo, int64_t hi, int64_t split,
                                double scale, torch::Tensor sq_local, int64_t max_blocks) {
  Group& g = get(gid);
  TT_CHECK(lo % 4 == 0 && hi % 4 == 0 && split % 4 == 0 && lo <= hi, "comm_rs: lo/hi/split must be multiples of 4");
  TT_CHECK(grad_offset % 256 == 0 && grad_offset + hi * 4 <= static_cast<int64_t>(g.bytes), "comm_rs: bad region");
  TT_CHECK(sq_local.is_cuda() && sq_local.scalar_type() == torch::kFloat32 && sq_local.numel() >= 2,
           "comm_rs: sq_local fp32 [2]");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  const uint64_t e0 = next_epoch(g);
  const int threads = 512;
  const int grid = std::max(1, std::min<int>(grid_for(g.device, std::max<long long>(1, (hi - lo) / 4), threads),
                                             static_cast<int>(max_blocks)));
  rs_sumsq_kernel<<<grid, threads, 0, cur_stream()>>>(table(g), static_cast<size_t>(grad_offset), lo, hi, split,
                                                       static_cast<float>(scale), g.emulated ? 0ull : e0, 0ull,
                                                       device_status_ptr(g.device), timeout_ns(),
                                                       sq_local.data_ptr<float>());
  TT_CUDA_CHECK(cudaGetLastError());
}

// Publish the total of per-bucket sums of squares (fp32 [n_buckets, 2]) to every peer's pad;
// returns the epoch the adamw_allgather calls of this step wait for.
int64_t comm_publish_sumsq(int64_t gid, torch::Tensor sq) {
  Group& g = get(gid);
  TT_CHECK(sq.is_cuda() && sq.scalar_type() == torch::kFloat32 && sq.is_contiguous() && sq.numel() % 2 == 0,
           "comm_publish_sumsq: fp32 [n, 2]");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  const uint64_t e = next_epoch(g);
  publish_sumsq_kernel<<<1, 32, 0, cur_stream()>>>(table(g), sq.data_ptr<float>(), static_cast<int>(sq.numel() / 2),
                                                  g.emulated ? 0ull : e);
  TT_CUDA_CHECK(cudaGetLastError());
  return static_cast<int64_t>(e);
}

// ZeRO-1: clip + AdamW on [lo, hi) + fp32 all-gather into every rank's buffer at data_offset.
// norm_out (fp32 [2], optional): global grad norm and the clip coefficient applied.
void comm_adamw_allgather(int64_t gid, int64_t data_offset, int64_t grad_offset, c10::optional<torch::Tensor> p16,
                          torch::Tensor m, torch::Tensor v, int64_t lo, int64_t hi, double lr, double beta1,
                          double beta2, double eps, double wd, int64_t step, double max_norm,
                          c10::optional<torch::Tensor> extra_sq, c10::optional<torch::Tensor> norm_out,
                          int64_t pads_epoch) {
  Group& g = get(gid);
  TT_CHECK(lo % 4 == 0 && hi % 4 == 0 && lo <= hi, "comm_adamw: lo/hi must be multiples of 4");
  TT_CHECK(m.scalar_type() == torch::kFloat32 && v.scalar_type() == torch::kFloat32 && m.numel() == hi - lo &&
               v.numel() == hi - lo && m.is_contiguous() && v.is_contiguous(),
           "comm_adamw: m/v must be fp32 [hi-lo]");
  TT_CHECK(reinterpret_cast<uintptr_t>(m.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(v.data_ptr()) % 16 == 0,
           "comm_adamw: m/v alignment");
  TT_CHECK(data_offset % 256 == 0 && grad_offset % 256 == 0, "comm_adamw: offsets must be 256-byte aligned");
  __nv_bfloat16* p16p = nullptr;
  if (p16.has_value()) {
    TT_CHECK(p16->scalar_type() == torch::kBFloat16 && p16->numel() >= hi && p16->is_contiguous() &&
                 reinterpret_cast<uintptr_t>(p16->data_ptr()) % 16 == 0,
             "comm_adamw: bf16 shadow must cover [0, hi)");
    p16p = reinterpret_cast<__nv_bfloat16*>(p16->data_ptr());
  }
  const float* xs = nullptr;
  if (extra_sq.has_value()) xs = extra_sq->data_ptr<float>();
  float* nout = nullptr;
  if (norm_out.has_value()) {
    TT_CHECK(norm_out->numel() >= 2 && norm_out->scalar_type() == torch::kFloat32, "comm_adamw: norm_out fp32 [2]");
    nout = norm_out->data_ptr<float>();
  }
  AdamArgs a;
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  a.max_norm = static_cast<float>(max_norm);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  // The pads were published with the reduce-scatter's second epoch (the current one), or,
  // for the bucketed path, with the epoch comm_publish_sumsq returned (pads_epoch).
  const uint64_t e_pads = pads_epoch >= 0 ? static_cast<uint64_t>(pads_epoch) : g.epoch;
  const uint64_t e_done = next_epoch(g);
  const int threads = 512;
  const int grid = grid_for(g.device, std::max<long long>(1, (hi - lo) / 4), threads);
  adamw_allgather_kernel<<<grid, threads, 0, cur_stream()>>>(
      table(g), static_cast<size_t>(data_offset), static_cast<size_t>(grad_offset), p16p, m.data_ptr<float>(),
      v.data_ptr<float>(), lo, hi, a, xs, nout, g.emulated ? 0ull : e_pads, g.emulated ? 0ull : e_done,
      device_status_ptr(g.device), timeout_ns());
  TT_CUDA_CHECK(cudaGetLastError());
}

// Waits for the all-gather (current epoch) and refreshes the bf16 shadow outside [lo, hi).
void comm_shadow_refresh(int64_t gid, int64_t data_offset, torch::Tensor p16, int64_t lo, int64_t hi) {
  Group& g = get(gid);
  TT_CHECK(p16.scalar_type() == torch::kBFloat16 && p16.is_contiguous() && p16.numel() % 4 == 0,
           "comm_shadow_refresh: bf16 shadow, numel multiple of 4");
  const long long n = p16.numel();
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  const int threads = 512;
  const int grid = grid_for(g.device, std::max<long long>(1, n / 4), threads);
  shadow_refresh_kernel<<<grid, threads, 0, cur_stream()>>>(
      table(g), static_cast<size_t>(data_offset), reinterpret_cast<__nv_bfloat16*>(p16.data_ptr()), lo, hi, n,
      g.emulated ? 0ull : g.epoch, device_status_ptr(g.device), timeout_ns());
  TT_CUDA_CHECK(cudaGetLastError());
}

// Replayable (CUDA-graph safe) all-reduce of `in` over the group: out = sum over ranks
// (root < 0) or out = root's `in` (root >= 0, a broadcast), plus `residual` if given.
// The two slots of slot_bytes each at slot_offset hold the published inputs.  bf16 or
// fp32, numel * element size a multiple of 16 bytes.  Emulated groups must be launched
// rank by rank with every rank's publish before any reduce (replay_publish/reduce below).
static void check_replay_args(const Group& g, int64_t slot_offset, int64_t slot_bytes, const torch::Tensor& x) {
  const long long bytes = x.numel() * static_cast<long long>(x.element_size());
  TT_CHECK(x.is_cuda() && x.is_contiguous() && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && bytes % 16 == 0,
           "comm_replay: tensors must be contiguous, 16-byte aligned, a multiple of 16 bytes");
  TT_CHECK(x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat32, "comm_replay: bf16 or fp32");
  TT_CHECK(bytes <= slot_bytes && slot_offset % 256 == 0 && slot_bytes % 256 == 0 &&
               slot_offset >= static_cast<int64_t>(kUserOff) &&
               slot_offset + 2 * slot_bytes <= static_cast<int64_t>(g.bytes),
           "comm_replay: slots outside the heap or too small");
}

void comm_replay_publish(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor in) {
  Group& g = get(gid);
  check_replay_args(g, slot_offset, slot_bytes, in);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  const long long bytes = in.numel() * static_cast<long long>(in.element_size());
  const int grid = std::min(grid_for(g.device, std::max<long long>(1, bytes / 16), 256), num_sms(g.device));
  replay_publish_kernel<<<grid, 256, 0, cur_stream()>>>(table(g), static_cast<size_t>(slot_offset), slot_bytes,
                                                        static_cast<const char*>(in.data_ptr()), bytes);
  TT_CUDA_CHECK(cudaGetLastError());
}

void comm_replay_reduce(int64_t gid, int64_t slot_offset, int64_t slot_bytes, torch::Tensor out,
                        c10::optional<torch::Tensor> residual, int64_t root) {
  Group& g = get(gid);
  check_replay_args(g, slot_offset, slot_bytes, out);
  TT_CHECK(root < g.world, "comm_replay: root out of range");
  const void* res = nullptr;
  if (residual.has_value()) {
    TT_CHECK(residual->scalar_type() == out.scalar_type() && residual->numel() == out.numel() &&
                 residual->is_contiguous() && reinterpret_cast<uintptr_t>(residual->data_ptr()) % 16 == 0,
             "comm_replay: residual must match out");
    res = residual->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g.device));
  const long long n = out.numel();
  const int grid = std::min(grid_for(g.device, std::max<long long>(1, n / 8), 256), num_sms(g.device));
  const PeerTable t = table(g);
  int* st = device_status_ptr(g.device);
  if (out.scalar_type() == torch::kBFloat16)
    replay_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, cur_stream()>>>(
        t, static_cast<size_t>(slot_offset), slot_bytes, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(res), n, static_cast<int>(root), st, timeout_ns());
  else
    replay_reduce_kernel<float><<<grid, 256, 0, cur_stream()>>>(
        t, static_cast<size_t>(slot_offset), slot_bytes, out.data_ptr<float>(), reinterpret_cast<const float*>(res), n,
        static_cast<int>(root), st, timeout_ns());
  TT_CUDA_CHECK(cudaGetLastError());
}

int64_t comm_epoch(int64_t gid) { return static_cast<int64_t>(get(gid).epoch); }

void comm_destroy(int64_t gid) {
  Group* g = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    TT_CHECK(gid >= 0 && gid < static_cast<int64_t>(g_groups.size()) && g_groups[gid] != nullptr,
             "comm: invalid group id");
    g = g_groups[gid];
    g_groups[gid] = nullptr;
  }
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(g->device));
  TT_CUDA_CHECK(cudaDeviceSynchronize());
  for (int p = 0; p < kMaxRanks; ++p)
    if (g->opened[p]) cudaIpcCloseMemHandle(g->peer[p]);
  cudaFree(g->heap);
  delete g;
}

PeerTable group_table(int64_t gid) { return table(get(gid)); }
uint64_t group_next_epoch(int64_t gid) { return next_epoch(get(gid)); }
bool group_emulated(int64_t gid) { return get(gid).emulated; }
int group_device(int64_t gid) { return get(gid).device; }
size_t group_bytes(int64_t gid) { return get(gid).bytes; }
uint64_t wait_timeout_ns() { return timeout_ns(); }
int grid_blocks(int device, long long work_items, int threads) { return grid_for(device, work_items, threads); }
void launch_peer_wait(const PeerTable& t, uint64_t e, int* status, cudaStream_t s) {
  barrier_kernel<<<1, 32, 0, s>>>(t, e, status, timeout_ns(), 0);
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace comm
}  // namespace tt
