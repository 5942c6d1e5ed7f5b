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

// One CTA per (split of 64 keys, kv head, sequence); G (q heads per kv head) is a template
// parameter so no register or instruction is spent on absent heads.  Every phase has at
// most one dependent round trip to memory, so a CTA's life is a few memory latencies and
// the many small CTAs (4x more than 256-key splits) keep HBM busy:
//   scores: two threads per key, each dotting alternate 16-byte pieces of the key's row
//           (all of the chunk's K loads in flight at once) with the G query heads held in
//           shared memory (16-byte broadcast reads), then one shuffle;
//   softmax: chunk max and sum per head (block reductions);
//   P.V:    each warp takes every 4th key; a lane owns D/32 dims, so a warp reads whole V
//           rows; 16 keys per warp = the whole chunk in one step, all loads in flight; the
//           4 warp partials are summed in warp order.  Key rows come from a per-chunk table
//           in shared memory filled during the score pass (one page-table lookup per key).
template <int D, int G>
__global__ void __launch_bounds__(kThreads, 4) decode_split_kernel(const DecodeParams p) {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(kChunk * 2 == kThreads, "two threads per key");
  constexpr int NV = D / 8;  // uint4 per K row
  constexpr int NW = kThreads / 32;
  constexpr int KPW = kChunk / NW;  // keys per warp in P.V
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int L = (p.len_dev != nullptr ? *p.len_dev : 0) + p.len_host;
  const int j0 = split * kChunk;
  const int n = max(0, min(kChunk, L - j0));
  __shared__ __align__(16) float q_s[G][D];
  __shared__ float s_s[G][kChunk];
  __shared__ float red_s[NW][G];
  __shared__ float m_s[G], l_s[G];
  __shared__ __align__(16) float o_s[NW][G][D];
  __shared__ long long rows_s[kChunk];  // page-pool row of each key of the chunk (-1: unmapped)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (n == 0) {  // split past the current length (uniform per CTA): an empty partial
    if (tid < G) {
      const long long rowo = (static_cast<long long>(b) * p.Hq + kvh * G + tid) * p.splits + split;
      p.ml_part[rowo * 2] = -INFINITY;
      p.ml_part[rowo * 2 + 1] = 0.f;
    }
    return;
  }
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    q_s[g][d] = __bfloat162float(p.q[(static_cast<long long>(b) * p.Hq + kvh * G + g) * D + d]);
  }
  __syncthreads();
  // ---- scores: thread pair (2j, 2j+1) takes key j; thread hh dots 16-byte pieces hh, hh+2, ...
  {
    const int j = tid >> 1, hh = tid & 1;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
    if (j < n) {
      const int key = j0 + j;
      const int pi = key / p.page_size;
      const int page = pi < p.pages_per_seq ? p.page_table[static_cast<long long>(b) * p.pages_per_seq + pi] : -1;
      const long long row =
          (page < 0 || page >= p.num_pages) ? -1ll : static_cast<long long>(page) * p.page_size + key % p.page_size;
      if (hh == 0) rows_s[j] = row;
      if (row >= 0) {
        const uint4* kr = reinterpret_cast<const uint4*>(p.k_pages + (row * p.Hkv + kvh) * D);
        uint4 kv[NV / 2];
#pragma unroll
        for (int c = 0; c < NV / 2; ++c) kv[c] = kr[2 * c + hh];
#pragma unroll
        for (int c = 0; c < NV / 2; ++c) {
          const int d0 = 8 * (2 * c + hh);
          const uint32_t* w = reinterpret_cast<const uint32_t*>(&kv[c]);
          float kf[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_bf16x2(w[e]);
            kf[2 * e] = f.x;
            kf[2 * e + 1] = f.y;
          }
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float4 qa = *reinterpret_cast<const float4*>(&q_s[g][d0]);
            const float4 qb = *reinterpret_cast<const float4*>(&q_s[g][d0 + 4]);
            acc[g] += kf[0] * qa.x + kf[1] * qa.y + kf[2] * qa.z + kf[3] * qa.w + kf[4] * qb.x + kf[5] * qb.y +
                      kf[6] * qb.z + kf[7] * qb.w;
          }
        }
      } else if (hh == 0) {
        atomicCAS(p.status, 0, static_cast<int>(kBadIndex));
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
    if (j < n && hh == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) s_s[g][j] = acc[g] * p.scale_log2;
    }
  }
  __syncthreads();
  // ---- chunk max per head (warp w < G reduces head w over the chunk)
  if (warp < G) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, s_s[warp][j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) m_s[warp] = m;
  }
  if constexpr (G > NW) {
    for (int g = NW + warp; g < G; g += NW) {
      float m = -INFINITY;
      for (int j = lane; j < n; j += 32) m = fmaxf(m, s_s[g][j]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) m_s[g] = m;
    }
  }
  __syncthreads();
  // ---- probabilities (in place) and their sums
  for (int g = warp; g < G; g += NW) {
    const float m = m_s[g];
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = exp2f(s_s[g][j] - m);
      s_s[g][j] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) l_s[g] = l;
  }
  __syncthreads();
  // ---- P.V: warp w takes keys w, w+4, ...; lane owns D/32 consecutive dims (one 8- or
  // 4-byte load per key, a warp reads whole V rows); the chunk in one step, all loads in flight.
  constexpr int DPL = D / 32;
  float oacc[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < DPL; ++e) oacc[g][e] = 0.f;
  {
    float vv[KPW][DPL];
#pragma unroll
    for (int u = 0; u < KPW; ++u) {
      const int j = warp + u * NW;
      const long long row = j < n ? rows_s[j] : -1;
      if (row >= 0) {
        const __nv_bfloat16* vr = p.v_pages + (row * p.Hkv + kvh) * D + lane * DPL;
        if constexpr (DPL == 4) {
          const uint2 w = *reinterpret_cast<const uint2*>(vr);
          const float2 a = unpack_bf16x2(w.x), c = unpack_bf16x2(w.y);
          vv[u][0] = a.x; vv[u][1] = a.y; vv[u][2] = c.x; vv[u][3] = c.y;
        } else {
          const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(vr));
          vv[u][0] = a.x; vv[u][1] = a.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) vv[u][e] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < KPW; ++u) {
      const int j = warp + u * NW;
      if (j < n) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pr = s_s[g][j];
#pragma unroll
          for (int e = 0; e < DPL; ++e) oacc[g][e] += pr * vv[u][e];
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int e = 0; e < DPL; ++e) o_s[warp][g][lane * DPL + e] = oacc[g][e];
  }
  __syncthreads();
  // sum the NW partitions in warp order: thread handles (g, d) pairs
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) o += o_s[w][g][d];
    const long long rowo = (static_cast<long long>(b) * p.Hq + kvh * G + g) * p.splits + split;
    p.o_part[rowo * D + d] = o;
    if (d == 0) {
      p.ml_part[rowo * 2] = n > 0 ? m_s[g] : -INFINITY;
      p.ml_part[rowo * 2 + 1] = n > 0 ? l_s[g] : 0.f;
    }
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
  TT_CHECK(q.dim() == 3 && q.is_contiguous(), "decode_attention: q must be [B, Hq, D]");
  const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2);
  TT_CHECK(k_pages.dim() == 4 && k_pages.size(3) == D && v_pages.sizes() == k_pages.sizes() &&
               k_pages.is_contiguous() && v_pages.is_contiguous(),
           "decode_attention: pages [num_pages, page_size, Hkv, D]");
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
#define TT_DECODE(DV, GV) decode::decode_split_kernel<DV, GV><<<grid, decode::kThreads, 0, cur_stream()>>>(p)
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
