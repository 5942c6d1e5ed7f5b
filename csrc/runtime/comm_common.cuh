// Shared pieces of the tt_comm runtime (csrc/runtime/comm.cu) used by every file
// whose kernels talk to peers through a symmetric heap: the heap layout, the peer
// table passed to kernels, bounded release/acquire signalling, and the host-side
// accessors of a group.
#pragma once
#include "common/ptx.cuh"
#include "common/host_utils.h"

namespace tt {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr size_t kFlagsOff = 0;
constexpr size_t kPadsOff = 1024;
constexpr int kPadFloats = 64;
constexpr size_t kCounterOff = 4096;
constexpr size_t kPartialOff = 8192;
constexpr int kMaxBlocks = 512;  // kPartialOff + kMaxBlocks * 4 floats fits below the user region
// Device-side epoch of the replayable collectives (local use only).  Kernels read it at
// their start and the last block of a collective's final kernel advances it, so a
// collective captured in a CUDA graph synchronises correctly on every replay (a host
// epoch baked into the graph would not).
constexpr size_t kDevEpochOff = 16384;
constexpr size_t kUserOff = 65536;

struct PeerTable {
  char* base[kMaxRanks];
  int rank;
  int world;
};

// ------------------------------------------------------------------ device helpers
__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t* flag_ptr(const PeerTable& t, int owner, int writer) {
  return reinterpret_cast<uint64_t*>(t.base[owner] + kFlagsOff) + writer;
}
__device__ __forceinline__ float* pad_ptr(const PeerTable& t, int owner, int writer) {
  return reinterpret_cast<float*>(t.base[owner] + kPadsOff) + writer * kPadFloats;
}

// One thread: publish epoch e to every peer (after everything this thread can see).
__device__ __forceinline__ void signal_peers(const PeerTable& t, uint64_t e) {
  __threadfence_system();
  for (int p = 0; p < t.world; ++p)
    if (p != t.rank) st_release_sys_u64(flag_ptr(t, p, t.rank), e);
  // Our own slot too, so a single-rank group (and the emulated test mode) is uniform.
  st_release_sys_u64(flag_ptr(t, t.rank, t.rank), e);
}

// Epoch of the next replayable collective step (the device-side counter + 1); the last
// kernel of the step stores it back (see kDevEpochOff).
__device__ __forceinline__ uint64_t dev_epoch_next(const PeerTable& t) {
  return *reinterpret_cast<volatile uint64_t*>(t.base[t.rank] + kDevEpochOff) + 1;
}

// One thread: wait until every peer published epoch >= e.  Bounded.
__device__ __forceinline__ bool wait_peers(const PeerTable& t, uint64_t e, int* status, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer();
  for (int p = 0; p < t.world; ++p) {
    if (p == t.rank) continue;
    const uint64_t* f = flag_ptr(t, t.rank, p);
    while (ld_acquire_sys_u64(f) < e) {
      if (status != nullptr && *reinterpret_cast<volatile int*>(status) != 0) return false;
      if (globaltimer() - t0 > timeout_ns) {
        if (status != nullptr) atomicCAS(status, 0, static_cast<int>(kTimeoutPeer));
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// All threads of the block: thread 0 waits, the verdict is broadcast.
__device__ __forceinline__ bool block_wait_peers(const PeerTable& t, uint64_t e, int* status, uint64_t timeout_ns) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) ok_s = wait_peers(t, e, status, timeout_ns) ? 1 : 0;
  __syncthreads();
  return ok_s != 0;
}

// All threads of the block, at the end of a kernel: the last block to arrive
// (after every block's global/peer stores are fenced) runs `last_fn` on thread 0.
template <typename F>
__device__ __forceinline__ void grid_last_block(const PeerTable& t, F last_fn) {
  __shared__ int last_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    unsigned int* counter = reinterpret_cast<unsigned int*>(t.base[t.rank] + kCounterOff);
    const unsigned int prev = atomicAdd(counter, 1u);
    last_s = (prev == gridDim.x - 1) ? 1 : 0;
    if (last_s) {
      __threadfence_system();
      *counter = 0u;  // ready for the next kernel (kernel boundaries order this)
      last_fn();
    }
  }
  __syncthreads();
}

// Deterministic block reduction of two floats (blockDim.x a multiple of 32, <= 1024).
__device__ __forceinline__ float2 block_sum2(float a, float b) {
  __shared__ float2 red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = make_float2(a, b);
  __syncthreads();
  float2 r = make_float2(0.f, 0.f);
  if (threadIdx.x == 0) {
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) {
      r.x += red[i].x;
      r.y += red[i].y;
    }
  }
  __syncthreads();
  return r;  // valid on thread 0
}

// ------------------------------------------------------------------ host accessors
// (implemented in comm.cu)
PeerTable group_table(int64_t gid);      // peer table of an opened group
uint64_t group_next_epoch(int64_t gid);  // advance and return the group's epoch
bool group_emulated(int64_t gid);        // single-GPU test mode (waits disabled)
int group_device(int64_t gid);
size_t group_bytes(int64_t gid);
uint64_t wait_timeout_ns();
int grid_blocks(int device, long long work_items, int threads);
// Launch a one-thread wait (no signal) for epoch e of every peer on stream s.
void launch_peer_wait(const PeerTable& t, uint64_t e, int* status, cudaStream_t s);

}  // namespace comm
}  // namespace tt
