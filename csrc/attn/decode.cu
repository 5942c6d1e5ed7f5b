// KV-cache decode path for sm_100a: fused RoPE + paged KV append, and split-KV
// ("flash-decoding") attention that reads K/V straight from the pages through the
// page table.  Both kernels take the sequence position from a device int32, so a
// whole decode step can be captured once in a CUDA graph and replayed.
//
// Replaces, for the reference's cached inference (tinytron/model/modules/attn.py:
// 188-224, 314-341, 420 and tinytron/inference/cache.py:34-51): the per-step RoPE
// recomputation (attn.py:13-63), the KV-cache copy_, the GQA expansion
// (attn.py:66-83), the boolean cache mask (attn.py:86-95) and SDPA over the
// concatenated cache.  K/V heads are stored unexpanded; one CTA serves all q heads
// of a kv head, so every K/V byte is read once per step.
//
// Decode attention is bound by K/V bytes (a few MB per layer), so the dot products
// run on the FMA pipe: two threads per key for the scores, and P·V with lanes owning
// output dims; small 64-key splits keep enough independent loads in flight.
#include "common/ptx.cuh"
#include "common/host_utils.h"

#include <mutex>
#include <type_traits>

namespace tt {
namespace decode {

constexpr int kChunk = 64;    // keys per split CTA
constexpr int kThreads = 128;
constexpr int kMaxG = 8;      // q heads per kv head
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- RoPE + append
// One thread per (token, head, 8-dim group of the first half): rotates dims
// [8c, 8c+8) together with [D/2 + 8c, D/2 + 8c + 8).  q heads -> q_out; k heads ->
// k pages (rotated); v heads -> v pages (copied).
__global__ void rope_append_kernel(const __nv_bfloat16* __restrict__ qkv, int ld, int B, int T, int Hq, int Hkv,
                                   int D, const int* __restrict__ pos_dev, int pos_host, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, int max_pos, __nv_bfloat16* __restrict__ q_out,
                                   __nv_bfloat16* __restrict__ k_pages, __nv_bfloat16* __restrict__ v_pages,
                                   const int* __restrict__ page_table, int pages_per_seq, int page_size,
                                   int num_pages, int* status) {
  const int groups = D / 16;  // 8-dim groups in the first half
  const int H = Hq + 2 * Hkv;
  const long long total = static_cast<long long>(B) * T * H * groups;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % groups);
  const int h = static_cast<int>((idx / groups) % H);
  const long long tok = idx / (static_cast<long long>(groups) * H);  // b * T + t
  const int b = static_cast<int>(tok / T);
  const int t = static_cast<int>(tok % T);
  const int pos = (pos_dev != nullptr ? *pos_dev : 0) + pos_host + t;
  if (pos < 0) {
    atomicCAS(status, 0, static_cast<int>(kBadIndex));
    return;
  }
  const __nv_bfloat16* src = qkv + tok * ld + static_cast<long long>(h) * D;
  const int d0 = 8 * c, d1 = D / 2 + 8 * c;
  const uint4 lo4 = *reinterpret_cast<const uint4*>(src + d0);
  const uint4 hi4 = *reinterpret_cast<const uint4*>(src + d1);
  uint4 olo = lo4, ohi = hi4;
  if (h < Hq + Hkv) {  // rotate q and k
    if (pos >= max_pos) {
      atomicCAS(status, 0, static_cast<int>(kBadIndex));
      return;
    }
    const float* cr = cos_t + static_cast<long long>(pos) * (D / 2) + d0;
    const float* sr = sin_t + static_cast<long long>(pos) * (D / 2) + d0;
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&lo4);
    const uint32_t* bb = reinterpret_cast<const uint32_t*>(&hi4);
    uint32_t* oa = reinterpret_cast<uint32_t*>(&olo);
    uint32_t* ob = reinterpret_cast<uint32_t*>(&ohi);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x1 = unpack_bf16x2(a[i]);
      const float2 x2 = unpack_bf16x2(bb[i]);
      const float c0 = cr[2 * i], c1 = cr[2 * i + 1], s0 = sr[2 * i], s1 = sr[2 * i + 1];
      // [x1, x2] -> [x1 cos - x2 sin, x2 cos + x1 sin]  (half-split rotation)
      oa[i] = pack_bf16x2(x1.x * c0 - x2.x * s0, x1.y * c1 - x2.y * s1);
      ob[i] = pack_bf16x2(x2.x * c0 + x1.x * s0, x2.y * c1 + x1.y * s1);
    }
  }
  __nv_bfloat16* dst;
  if (h < Hq) {
    dst = q_out + tok * static_cast<long long>(Hq) * D + static_cast<long long>(h) * D;
  } else {
    const int kvh = (h < Hq + Hkv) ? h - Hq : h - Hq - Hkv;
    const int pi = pos / page_size;
    if (pi >= pages_per_seq) {
      atomicCAS(status, 0, static_cast<int>(kBadIndex));
      return;
    }
    const int page = page_table[static_cast<long long>(b) * pages_per_seq + pi];
    if (page < 0 || page >= num_pages) {
      atomicCAS(status, 0, static_cast<int>(kBadIndex));
      return;
    }
    __nv_bfloat16* pages = (h < Hq + Hkv) ? k_pages : v_pages;
    dst = pages + ((static_cast<long long>(page) * page_size + pos % page_size) * Hkv + kvh) * D;
  }
  *reinterpret_cast<uint4*>(dst + d0) = olo;
  *reinterpret_cast<uint4*>(dst + d1) = ohi;
}

// ---------------------------------------------------------------- split-KV attention
struct DecodeParams {
  const __nv_bfloat16* q;        // [B, Hq, D] (one new token per sequence)
  const __nv_bfloat16* k_pages;  // [num_pages, page_size, Hkv, D]
  const __nv_bfloat16* v_pages;
  const int* page_table;         // [B, pages_per_seq]
  const int* len_dev;            // optional: keys = *len_dev + len_host
  int len_host;
  int B, Hq, Hkv, D;
  int pages_per_seq, page_size, num_pages;
  int splits;
  float scale_log2;              // softmax scale * log2(e)
  float* o_part;                 // [B, Hq, splits, D] unnormalised
  float* ml_part;                // [B, Hq, splits, 2] (running max in log2 units, sum)
  int* status;
};

// 16-byte global -> shared copy without registers (LDGSTS); zero-fills when !valid.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
// Four 8x8 bf16 matrices from shared memory (row addresses from lanes 0-7, 8-15, 16-23, 24-31).
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
// c[16x8] += a[16x16] b[16x8], bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kRowPad = 8;  // bf16 padding per shared row: the 8 rows of an ldmatrix hit distinct banks

// One CTA per (split of 64 keys, kv head, sequence); G (q heads per kv head) is a template
// parameter.  A CTA's life is two dependent trips to memory, so the many small CTAs keep
// HBM busy:
//   1. the page-pool row of every key of the chunk (one page-table lookup per key, into
//      shared memory) and the G query heads (asynchronous copies);
//   2. the chunk's K and V rows (32 KB at D = 128), all in flight at once as 16-byte
//      asynchronous copies into padded shared rows (keys past the length read as zeros).
// The two products run on the tensor cores as 16x8x16 warp MMAs with the G query heads as
// the rows of a 16-row tile (rows >= G are never read back, so they need no zeroing):
//   S = Q K^T: warp w takes keys [16w, 16w + 16) over all of D;
//   softmax:   warp w owns heads w, w + 4, ...: chunk max, 2^(s - m) rounded to bf16 (the
//              P operand) and the sum of the rounded values;
//   O = P V:   warp w takes dims [wD/4, (w+1)D/4) over the 64 keys (V through transposing
//              ldmatrix), so each output element has exactly one owner and no partials
//              are summed.
// A warp MMA is the right size here: the M side is G <= 8 heads, below the 64-row minimum
// of a tcgen05 tile, and the kernel is bound by the K/V bytes, not by tensor throughput.
template <int D, int G>
__global__ void __launch_bounds__(kThreads, 4) decode_split_kernel(const DecodeParams p) {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(G <= 8, "at most 8 q heads per kv head (one 16-row tile, upper half unused)");
  constexpr int NV = D / 8;          // 16-byte pieces per row
  constexpr int RS = D + kRowPad;    // shared K/V/Q row stride (bf16)
  constexpr int PS = kChunk + kRowPad;
  constexpr int NW = kThreads / 32;
  static_assert(NW * 16 == kChunk, "one 16-key slice per warp");
  constexpr int DW = D / NW;         // output dims per warp
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int L = (p.len_dev != nullptr ? *p.len_dev : 0) + p.len_host;
  const int j0 = split * kChunk;
  const int n = max(0, min(kChunk, L - j0));
  __shared__ __align__(16) __nv_bfloat16 k_s[kChunk][RS];
  __shared__ __align__(16) __nv_bfloat16 v_s[kChunk][RS];
  __shared__ __align__(16) __nv_bfloat16 q_s[16][RS];
  __shared__ __align__(16) __nv_bfloat16 p_s[16][PS];
  __shared__ float s_s[G][kChunk];
  __shared__ float m_s[G], l_s[G];
  __shared__ long long rows_s[kChunk];  // page-pool row of each key of the chunk (-1: none)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (n == 0) {  // split past the current length (uniform per CTA): an empty partial
    if (tid < G) {
      const long long rowo = (static_cast<long long>(b) * p.Hq + kvh * G + tid) * p.splits + split;
      p.ml_part[rowo * 2] = -INFINITY;
      p.ml_part[rowo * 2 + 1] = 0.f;
    }
    return;
  }
  // ---- trip 1: key rows and query heads
  if (tid < kChunk) {
    long long row = -1;
    if (tid < n) {
      const int key = j0 + tid;
      const int pi = key / p.page_size;
      const int page = pi < p.pages_per_seq ? p.page_table[static_cast<long long>(b) * p.pages_per_seq + pi] : -1;
      if (page >= 0 && page < p.num_pages) row = static_cast<long long>(page) * p.page_size + key % p.page_size;
      else atomicCAS(p.status, 0, static_cast<int>(kBadIndex));
    }
    rows_s[tid] = row;
  }
  const __nv_bfloat16* qg = p.q + (static_cast<long long>(b) * p.Hq + kvh * G) * D;
  for (int i = tid; i < G * NV; i += kThreads) cp_async16(&q_s[i / NV][8 * (i % NV)], qg + 8 * i, true);
  cp_async_wait_all();
  __syncthreads();
  // ---- trip 2: the chunk's K and V rows (consecutive threads copy consecutive pieces of a row)
#pragma unroll 4
  for (int i = tid; i < kChunk * NV; i += kThreads) {
    const int r = i / NV, c = i % NV;
    const long long row = rows_s[r];
    const long long off = row >= 0 ? (row * p.Hkv + kvh) * D + 8 * c : 0;
    cp_async16(&k_s[r][8 * c], p.k_pages + off, row >= 0);
    cp_async16(&v_s[r][8 * c], p.v_pages + off, row >= 0);
  }
  cp_async_wait_all();
  __syncthreads();
  const int lr = lane & 7, lm = lane >> 3;  // row within an 8x8 matrix, matrix index
  // ---- S = Q K^T for keys [16w, 16w + 16)
  {
    float sacc[2][4] = {};
    const int kb = warp * 16;
#pragma unroll
    for (int k0 = 0; k0 < D; k0 += 16) {
      uint32_t a[4], bk[4];
      ldsm_x4(a, &q_s[lane & 15][k0 + (lane >> 4) * 8]);
      // matrices: (keys kb..+7, dims k0..+7), (kb..+7, k0+8..), (kb+8..+15, k0..), (kb+8.., k0+8..)
      ldsm_x4(bk, &k_s[kb + (lm >> 1) * 8 + lr][k0 + (lm & 1) * 8]);
      mma_bf16_16816(sacc[0], a, bk[0], bk[1]);
      mma_bf16_16816(sacc[1], a, bk[2], bk[3]);
    }
    const int g = lane >> 2;
    if (g < G) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int j = kb + t * 8 + 2 * (lane & 3);
        s_s[g][j] = sacc[t][0] * p.scale_log2;
        s_s[g][j + 1] = sacc[t][1] * p.scale_log2;
      }
    }
  }
  __syncthreads();
  // ---- softmax of the chunk per head: P (bf16, zero past the length) and its sum
  for (int g = warp; g < G; g += NW) {
    float m = -INFINITY;
    for (int jj = lane; jj < n; jj += 32) m = fmaxf(m, s_s[g][jj]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
#pragma unroll
    for (int jj = lane; jj < kChunk; jj += 32) {
      const __nv_bfloat16 e = __float2bfloat16_rn(jj < n ? exp2f(s_s[g][jj] - m) : 0.f);
      p_s[g][jj] = e;
      l += __bfloat162float(e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      m_s[g] = m;
      l_s[g] = l;
    }
  }
  __syncthreads();
  // ---- O = P V for dims [w DW, (w + 1) DW)
  {
    constexpr int NT = DW / 8;  // 8-dim n-tiles per warp
    static_assert(NT % 2 == 0, "n-tiles are loaded in pairs");
    float oacc[NT][4] = {};
    const int db = warp * DW;
#pragma unroll
    for (int k0 = 0; k0 < kChunk; k0 += 16) {
      uint32_t a[4];
      ldsm_x4(a, &p_s[lane & 15][k0 + (lane >> 4) * 8]);
#pragma unroll
      for (int t = 0; t < NT; t += 2) {
        uint32_t bv[4];
        // matrices: (keys k0..+7, dims t), (k0+8..+15, dims t), (k0..+7, dims t+1), (k0+8.., dims t+1)
        ldsm_x4_t(bv, &v_s[k0 + (lm & 1) * 8 + lr][db + (t + (lm >> 1)) * 8]);
        mma_bf16_16816(oacc[t], a, bv[0], bv[1]);
        mma_bf16_16816(oacc[t + 1], a, bv[2], bv[3]);
      }
    }
    const int g = lane >> 2;
    if (g < G) {
      const long long rowo = (static_cast<long long>(b) * p.Hq + kvh * G + g) * p.splits + split;
      float* o = p.o_part + rowo * D + db + 2 * (lane & 3);
#pragma unroll
      for (int t = 0; t < NT; ++t) *reinterpret_cast<float2*>(o + t * 8) = make_float2(oacc[t][0], oacc[t][1]);
    }
  }
  if (tid < G) {
    const long long rowo = (static_cast<long long>(b) * p.Hq + kvh * G + tid) * p.splits + split;
    p.ml_part[rowo * 2] = m_s[tid];
    p.ml_part[rowo * 2 + 1] = l_s[tid];
  }
}

// out[b, h, :] = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s
__global__ void decode_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ ml_part, int splits,
                                      int D, __nv_bfloat16* __restrict__ out) {
  const long long row = blockIdx.x;  // b * Hq + h
  const float* ml = ml_part + row * splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ml[2 * s]);
  float den = 0.f;
  for (int s = 0; s < splits; ++s)
    if (ml[2 * s + 1] > 0.f) den += exp2f(ml[2 * s] - M) * ml[2 * s + 1];
  const float inv = den > 0.f ? 1.0f / den : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s)
      if (ml[2 * s + 1] > 0.f) acc += exp2f(ml[2 * s] - M) * o_part[(row * splits + s) * D + d];
    out[row * D + d] = __float2bfloat16_rn(acc * inv);
  }
}

// The split kernel's ~40 KB of static shared memory allows 5 CTAs per SM only with the
// largest shared-memory carveout, so ask for it (a per-kernel attribute, set once).
template <int D, int G>
void launch_split(const DecodeParams& p, dim3 grid, cudaStream_t stream, int device) {
  static std::once_flag once[64];  // the attribute belongs to the current device's context
  std::call_once(once[device & 63], [] {
    cudaFuncSetAttribute(decode_split_kernel<D, G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
  });
  decode_split_kernel<D, G><<<grid, kThreads, 0, stream>>>(p);
}

}  // namespace decode

// qkv [B*T, ld] bf16 (q | k | v heads, D each) -> q_out [B*T, Hq*D] rotated; K/V
// (k rotated) appended at positions (*pos_dev + pos_host + t) into the pages.
void decode_rope_append(torch::Tensor qkv, int64_t B, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                        c10::optional<torch::Tensor> pos_dev, int64_t pos_host, torch::Tensor cos_t,
                        torch::Tensor sin_t, torch::Tensor q_out, torch::Tensor k_pages, torch::Tensor v_pages,
                        torch::Tensor page_table) {
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(q_out, "q_out");
  check_cuda_bf16(k_pages, "k_pages");
  check_cuda_bf16(v_pages, "v_pages");
  TT_CHECK(D % 16 == 0 && D <= 256, "decode_rope_append: head_dim must be a multiple of 16");
  TT_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(0) == B * T && qkv.size(1) >= (Hq + 2 * Hkv) * D &&
               qkv.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0,
           "decode_rope_append: qkv must be [B*T, >=(Hq+2Hkv)*D], 16-byte aligned rows");
  TT_CHECK(q_out.is_contiguous() && q_out.numel() == B * T * Hq * D, "decode_rope_append: q_out [B*T, Hq*D]");
  TT_CHECK(k_pages.dim() == 4 && k_pages.size(2) == Hkv && k_pages.size(3) == D && k_pages.is_contiguous() &&
               v_pages.sizes() == k_pages.sizes() && v_pages.is_contiguous(),
           "decode_rope_append: pages must be [num_pages, page_size, Hkv, D]");
  TT_CHECK(page_table.scalar_type() == torch::kInt32 && page_table.dim() == 2 && page_table.size(0) == B &&
               page_table.is_contiguous(),
           "decode_rope_append: page_table int32 [B, pages_per_seq]");
  TT_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.size(1) == D / 2 && sin_t.sizes() == cos_t.sizes(),
           "decode_rope_append: cos/sin fp32 [max_pos, D/2]");
  const int* pd = nullptr;
  if (pos_dev.has_value()) {
    TT_CHECK(pos_dev->scalar_type() == torch::kInt32 && pos_dev->is_cuda(), "pos_dev must be a CUDA int32 scalar");
    pd = pos_dev->data_ptr<int>();
  }
  const long long total = B * T * (Hq + 2 * Hkv) * (D / 16);
  if (total == 0) return;
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int threads = 256;
  decode::rope_append_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), static_cast<int>(qkv.stride(0)), static_cast<int>(B),
      static_cast<int>(T), static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(D), pd,
      static_cast<int>(pos_host), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), static_cast<int>(cos_t.size(0)),
      reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), reinterpret_cast<__nv_bfloat16*>(k_pages.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v_pages.data_ptr()), page_table.data_ptr<int>(),
      static_cast<int>(page_table.size(1)), static_cast<int>(k_pages.size(1)), static_cast<int>(k_pages.size(0)),
      device_status_ptr(qkv.get_device()));
  TT_CUDA_CHECK(cudaGetLastError());
}

int64_t decode_num_splits(int64_t max_len) { return (max_len + decode::kChunk - 1) / decode::kChunk; }

// Attention of one new token per sequence over keys [0, L), L = *len_dev + len_host
// (<= splits * 256).  o_part/ml_part: fp32 scratch [B*Hq*splits*D], [B*Hq*splits*2].
void decode_attention(torch::Tensor q, torch::Tensor k_pages, torch::Tensor v_pages, torch::Tensor page_table,
                      c10::optional<torch::Tensor> len_dev, int64_t len_host, int64_t splits, double scale,
                      torch::Tensor o_part, torch::Tensor ml_part, torch::Tensor out) {
  check_cuda_bf16(q, "q");
  check_cuda_bf16(out, "out");
  TT_CHECK(q.dim() == 3 && q.is_contiguous() && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
           "decode_attention: q must be a 16-byte aligned contiguous [B, Hq, D]");
  const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2);
  TT_CHECK(k_pages.dim() == 4 && k_pages.size(3) == D && v_pages.sizes() == k_pages.sizes() &&
               k_pages.is_contiguous() && v_pages.is_contiguous() &&
               reinterpret_cast<uintptr_t>(k_pages.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(v_pages.data_ptr()) % 16 == 0,
           "decode_attention: pages [num_pages, page_size, Hkv, D], 16-byte aligned");
  const int64_t Hkv = k_pages.size(2);
  TT_CHECK(Hq % Hkv == 0 && Hq / Hkv <= decode::kMaxG, "decode_attention: Hq/Hkv must be an integer <= 8");
  TT_CHECK((Hq / Hkv) == 1 || (Hq / Hkv) == 2 || (Hq / Hkv) == 4 || (Hq / Hkv) == 8,
           "decode_attention: Hq/Hkv must be 1, 2, 4 or 8");
  TT_CHECK(D == 64 || D == 128, "decode_attention: head_dim 64 or 128");
  TT_CHECK(page_table.scalar_type() == torch::kInt32 && page_table.dim() == 2 && page_table.size(0) == B &&
               page_table.is_contiguous(),
           "decode_attention: page_table int32 [B, pages_per_seq]");
  TT_CHECK(splits >= 1 && splits * decode::kChunk >= 1, "decode_attention: splits >= 1");
  TT_CHECK(o_part.scalar_type() == torch::kFloat32 && o_part.numel() >= B * Hq * splits * D &&
               ml_part.scalar_type() == torch::kFloat32 && ml_part.numel() >= B * Hq * splits * 2,
           "decode_attention: scratch too small");
  TT_CHECK(out.is_contiguous() && out.numel() == B * Hq * D, "decode_attention: out [B, Hq*D]");
  decode::DecodeParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k_pages = reinterpret_cast<const __nv_bfloat16*>(k_pages.data_ptr());
  p.v_pages = reinterpret_cast<const __nv_bfloat16*>(v_pages.data_ptr());
  p.page_table = page_table.data_ptr<int>();
  p.len_dev = nullptr;
  if (len_dev.has_value()) {
    TT_CHECK(len_dev->scalar_type() == torch::kInt32 && len_dev->is_cuda(), "len_dev must be a CUDA int32 scalar");
    p.len_dev = len_dev->data_ptr<int>();
  }
  p.len_host = static_cast<int>(len_host);
  p.B = static_cast<int>(B);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.D = static_cast<int>(D);
  p.pages_per_seq = static_cast<int>(page_table.size(1));
  p.page_size = static_cast<int>(k_pages.size(1));
  p.num_pages = static_cast<int>(k_pages.size(0));
  p.splits = static_cast<int>(splits);
  p.scale_log2 = static_cast<float>(scale) * decode::kLog2e;
  p.o_part = o_part.data_ptr<float>();
  p.ml_part = ml_part.data_ptr<float>();
  p.status = device_status_ptr(q.get_device());
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(Hkv), static_cast<unsigned>(B));
  const int G = static_cast<int>(Hq / Hkv);
#define TT_DECODE(DV, GV) decode::launch_split<DV, GV>(p, grid, cur_stream(), q.get_device())
  if (D == 128) {
    switch (G) {
      case 1: TT_DECODE(128, 1); break;
      case 2: TT_DECODE(128, 2); break;
      case 4: TT_DECODE(128, 4); break;
      case 8: TT_DECODE(128, 8); break;
      default: TT_CHECK(false, "decode_attention: Hq/Hkv must be 1, 2, 4 or 8");
    }
  } else {
    switch (G) {
      case 1: TT_DECODE(64, 1); break;
      case 2: TT_DECODE(64, 2); break;
      case 4: TT_DECODE(64, 4); break;
      case 8: TT_DECODE(64, 8); break;
      default: TT_CHECK(false, "decode_attention: Hq/Hkv must be 1, 2, 4 or 8");
    }
  }
#undef TT_DECODE
  TT_CUDA_CHECK(cudaGetLastError());
  decode::decode_combine_kernel<<<static_cast<unsigned>(B * Hq), static_cast<unsigned>(D), 0, cur_stream()>>>(
      p.o_part, p.ml_part, p.splits, p.D, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
