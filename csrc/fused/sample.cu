// Token sampling for decode: temperature, top-k, top-p (nucleus) and the multinomial
// draw in one kernel per step, one CTA per sequence.
//
// Replaces the reference's sampler (tinytron/inference/sampler.py:6-61: topk, sort,
// softmax, cumsum, scatter, multinomial as separate library kernels).  Semantics kept:
//   * logits / temperature;
//   * top-k keeps every logit >= the k-th largest (ties included);
//   * top-p keeps the longest prefix of the probability-sorted tokens whose cumulative
//     mass is <= top_p, and always the most likely token;
//   * the token is drawn from the renormalised kept distribution; its log-probability
//     under that distribution is returned; top_k == 1 is the argmax (lowest index on ties).
// Thresholds come from radix selection over order-preserving 32-bit keys of the logits
// (four 8-bit digit passes with block histograms of counts or of probability mass), so
// nothing is sorted.  The uniform draw uses curand's Philox generator, seeded per call.
#include "common/host_utils.h"
#include "common/ptx.cuh"

#include <curand_kernel.h>

namespace tt {
namespace sample {

constexpr int THREADS = 1024;

__device__ __forceinline__ uint32_t key_of(float x) {  // monotone: a < b  <=>  key(a) < key(b)
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
__device__ __forceinline__ float load_logit(const T* row, int i, float inv_t) {
  return static_cast<float>(row[i]) * inv_t;
}

// Block reductions over THREADS threads (result broadcast to all threads).
__device__ __forceinline__ float block_max(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = sh[l];
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) sh[32] = v;
  }
  __syncthreads();
  return sh[32];
}
__device__ __forceinline__ float block_sum(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = sh[l];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) sh[32] = v;
  }
  __syncthreads();
  return sh[32];
}

// Radix select.  MODE 0: the key of the k-th largest element (count histogram).
// MODE 1: the largest key K such that the mass of keys > K is <= budget and the mass of
// keys >= K exceeds it (keys > K are the nucleus); returns 0 when everything fits.
// Each pass builds a 256-bin histogram of the next key byte: every warp adds into its own
// histogram (logits cluster in a few exponent bins, so one shared histogram would
// serialise all the block's atomics on those bins), 256 threads merge the 32 warp
// histograms, and a suffix scan over the bins picks the byte in one step.
constexpr int kWarps = THREADS / 32;

template <int MODE, typename T>
__device__ uint32_t radix_select(const T* row, int V, float inv_t, float mx, uint32_t floor_key, float target,
                                 float (*hist_w)[256], float* suf, float* sh) {
  uint32_t prefix = 0, prefix_mask = 0;
  float above = 0.0f;  // count / mass of keys strictly above the current prefix range
  const int warp = threadIdx.x >> 5;
  bool all_fit = false;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < kWarps * 256; i += THREADS) hist_w[i >> 8][i & 255] = 0.0f;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += THREADS) {
      const float x = load_logit(row, i, inv_t);
      const uint32_t k = key_of(x);
      if (k < floor_key || (k & prefix_mask) != prefix) continue;
      atomicAdd(&hist_w[warp][(k >> shift) & 0xFFu], MODE == 0 ? 1.0f : __expf(x - mx));
    }
    __syncthreads();
    // merge, then suffix sums from the top bin down (Hillis-Steele over 256 entries)
    if (threadIdx.x < 256) {
      float v = 0.0f;
#pragma unroll 8
      for (int w = 0; w < kWarps; ++w) v += hist_w[w][threadIdx.x];
      suf[threadIdx.x] = v;
    }
    __syncthreads();
    for (int o = 1; o < 256; o <<= 1) {
      float add = 0.0f;
      if (threadIdx.x < 256 && threadIdx.x + o < 256) add = suf[threadIdx.x + o];
      __syncthreads();
      if (threadIdx.x < 256) suf[threadIdx.x] += add;
      __syncthreads();
    }
    // the byte d: the highest bin whose cumulative count/mass from the top reaches the target
    if (threadIdx.x == 0) sh[33] = -1.0f;
    __syncthreads();
    if (threadIdx.x < 256) {
      const int d = threadIdx.x;
      const float incl = above + suf[d];
      const float excl = above + (d < 255 ? suf[d + 1] : 0.0f);
      const bool reach = MODE == 0 ? incl >= target : incl > target;
      const bool before = MODE == 0 ? excl >= target : excl > target;
      if (reach && !before) {
        sh[33] = static_cast<float>(d);
        sh[34] = excl;
      }
    }
    __syncthreads();
    const float dsel = sh[33];
    if (dsel < 0.0f) {  // everything left fits the budget (top-p keeps all candidates)
      all_fit = true;
      break;
    }
    above = sh[34];
    prefix |= static_cast<uint32_t>(dsel) << shift;
    prefix_mask |= 0xFFu << shift;
    __syncthreads();
  }
  __syncthreads();
  return all_fit ? 0u : prefix;
}

template <typename T>
__global__ void __launch_bounds__(THREADS) sample_kernel(const T* __restrict__ logits, int V, long long ld,
                                                        float inv_t, int top_k, float top_p,
                                                        unsigned long long seed, unsigned long long offset,
                                                        const long long* __restrict__ rng,
                                                        int64_t* __restrict__ tokens, float* __restrict__ logprob) {
  __shared__ float sh[36];
  __shared__ float hist_w[kWarps][256];
  __shared__ float suf[256];
  __shared__ float scan[THREADS];
  const int r = blockIdx.x;
  const T* row = logits + static_cast<long long>(r) * ld;
  // ---- max (and its lowest index for the greedy case)
  float mx = -INFINITY;
  int arg = V;
  for (int i = threadIdx.x; i < V; i += THREADS) {
    const float x = load_logit(row, i, inv_t);
    if (x > mx) {
      mx = x;
      arg = i;
    }
  }
  const float gmax = block_max(mx, sh);
  int cand = (mx == gmax) ? arg : V;
  for (int o = 16; o > 0; o >>= 1) cand = min(cand, __shfl_xor_sync(0xffffffffu, cand, o));
  __shared__ int amin[32];
  if ((threadIdx.x & 31) == 0) amin[threadIdx.x >> 5] = cand;
  __syncthreads();
  if (threadIdx.x == 0) {
    int a = V;
    for (int w = 0; w < THREADS / 32; ++w) a = min(a, amin[w]);
    amin[0] = a;
  }
  __syncthreads();
  const int argmax = amin[0];
  // ---- top-k threshold (keys >= kth are kept)
  uint32_t floor_key = 0;
  if (top_k == 1) {
    floor_key = key_of(gmax);
  } else if (top_k > 0 && top_k < V) {
    floor_key = radix_select<0>(row, V, inv_t, gmax, 0u, static_cast<float>(top_k), hist_w, suf, sh);
  }
  // ---- mass of the top-k set
  float z = 0.0f;
  for (int i = threadIdx.x; i < V; i += THREADS) {
    const float x = load_logit(row, i, inv_t);
    if (key_of(x) >= floor_key) z += __expf(x - gmax);
  }
  z = block_sum(z, sh);
  // ---- top-p: keys strictly above the nucleus threshold (always keeping the max)
  uint32_t excl = 0;  // 0: no top-p cut
  bool use_excl = false;
  if (top_k != 1 && top_p > 0.0f && top_p < 1.0f) {
    excl = radix_select<1>(row, V, inv_t, gmax, floor_key, top_p * z, hist_w, suf, sh);
    use_excl = true;
  }
  auto kept = [&](uint32_t k, int i) {
    if (k < floor_key) return false;
    if (use_excl && k <= excl && i != argmax) return false;
    return true;
  };
  // ---- kept mass and the draw
  const int chunk = (V + THREADS - 1) / THREADS;
  const int i0 = threadIdx.x * chunk, i1 = min(V, i0 + chunk);
  float part = 0.0f;
  for (int i = i0; i < i1; ++i) {
    const float x = load_logit(row, i, inv_t);
    if (kept(key_of(x), i)) part += __expf(x - gmax);
  }
  scan[threadIdx.x] = part;
  __syncthreads();
  for (int o = 1; o < THREADS; o <<= 1) {  // inclusive scan (Hillis-Steele), fixed order
    const float add = threadIdx.x >= o ? scan[threadIdx.x - o] : 0.0f;
    __syncthreads();
    scan[threadIdx.x] += add;
    __syncthreads();
  }
  const float zk = scan[THREADS - 1];
  __shared__ int64_t picked;
  if (threadIdx.x == 0) {
    picked = argmax;
    if (top_k != 1) {
      curandStatePhilox4_32_10_t st;
      if (rng != nullptr) {  // seed and offset from the device (a captured decode step)
        seed = static_cast<unsigned long long>(rng[0]);
        offset = static_cast<unsigned long long>(rng[1]);
      }
      curand_init(seed, static_cast<unsigned long long>(r), offset, &st);
      sh[34] = curand_uniform(&st) * zk;  // (0, zk]
    } else {
      sh[34] = -1.0f;
    }
  }
  __syncthreads();
  const float target = sh[34];
  if (target >= 0.0f) {
    const float before = threadIdx.x > 0 ? scan[threadIdx.x - 1] : 0.0f;
    if (target > before && target <= scan[threadIdx.x]) {
      float acc = before;
      int last = -1;
      for (int i = i0; i < i1; ++i) {
        const float x = load_logit(row, i, inv_t);
        if (!kept(key_of(x), i)) continue;
        last = i;
        acc += __expf(x - gmax);
        if (acc >= target) break;
      }
      if (last >= 0) picked = last;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    tokens[r] = picked;
    if (logprob != nullptr) {
      const float x = load_logit(row, static_cast<int>(picked), inv_t);
      logprob[r] = (x - gmax) - logf(top_k == 1 ? z : zk);
    }
  }
}

// One decode step's bookkeeping on the device, so that sampling and the next step's input
// live inside the captured decode graph: tokens[b, P + step] = nxt[b], the graph's token
// input = nxt, the log-prob into column `step`, then step += 1 (rng[1] is the step and the
// Philox offset of the next draw).  One block of B threads.  A step past the last column
// of `tokens` (total columns) or of `lp_all` (lp_cols) is not written and sets kBadIndex:
// the step lives on the device, so the host cannot bound it before the launch.
__global__ void decode_advance_kernel(const int64_t* __restrict__ nxt, int B, int64_t* __restrict__ tokens,
                                      long long ld_tokens, int P, long long total, int64_t* __restrict__ tok_in,
                                      long long* __restrict__ rng, const float* __restrict__ lp,
                                      float* __restrict__ lp_all, long long ld_lp, long long lp_cols,
                                      int* __restrict__ status) {
  const long long step = rng[1];
  const bool tok_ok = step >= 0 && P + step < total;
  const bool lp_ok = step >= 0 && step < lp_cols;
  if (threadIdx.x == 0 && (!tok_ok || (lp != nullptr && !lp_ok))) atomicCAS(status, 0, static_cast<int>(kBadIndex));
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int64_t t = nxt[b];
    if (tok_ok) tokens[b * ld_tokens + P + step] = t;
    tok_in[b] = t;
    if (lp != nullptr && lp_ok) lp_all[b * ld_lp + step] = lp[b];
  }
  __syncthreads();
  if (threadIdx.x == 0) rng[1] = step + 1;
}

}  // namespace sample

void decode_advance(torch::Tensor nxt, torch::Tensor tokens, int64_t P, torch::Tensor tok_in, torch::Tensor rng,
                    c10::optional<torch::Tensor> lp, c10::optional<torch::Tensor> lp_all) {
  TT_CHECK(nxt.is_cuda() && nxt.scalar_type() == torch::kInt64 && nxt.is_contiguous(), "decode_advance: nxt int64");
  const int64_t B = nxt.numel();
  TT_CHECK(tokens.is_cuda() && tokens.get_device() == nxt.get_device() && tokens.scalar_type() == torch::kInt64 &&
               tokens.dim() == 2 && tokens.size(0) == B && tokens.stride(1) == 1 && P >= 0 && P < tokens.size(1),
           "decode_advance: tokens int64 [B, total] on nxt's device, 0 <= P < total");
  TT_CHECK(tok_in.is_cuda() && tok_in.get_device() == nxt.get_device() && tok_in.scalar_type() == torch::kInt64 &&
               tok_in.numel() == B && tok_in.is_contiguous(),
           "decode_advance: token input int64 [B] on nxt's device");
  TT_CHECK(rng.scalar_type() == torch::kInt64 && rng.numel() >= 2 && rng.is_cuda() && rng.is_contiguous() &&
               rng.get_device() == nxt.get_device(),
           "decode_advance: rng int64 [2] on nxt's device");
  TT_CHECK(lp.has_value() == lp_all.has_value(), "decode_advance: lp and lp_all together");
  if (lp.has_value())
    TT_CHECK(lp->is_cuda() && lp_all->is_cuda() && lp->get_device() == nxt.get_device() &&
                 lp_all->get_device() == nxt.get_device() && lp->scalar_type() == torch::kFloat32 &&
                 lp->is_contiguous() && lp->numel() == B && lp_all->scalar_type() == torch::kFloat32 &&
                 lp_all->dim() == 2 && lp_all->size(0) == B && lp_all->stride(1) == 1,
             "decode_advance: lp fp32 [B], lp_all fp32 [B, steps] on nxt's device");
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(nxt.device());
  sample::decode_advance_kernel<<<1, static_cast<unsigned>(std::min<int64_t>(1024, ((B + 31) / 32) * 32)), 0,
                                  cur_stream()>>>(
      nxt.data_ptr<int64_t>(), static_cast<int>(B), tokens.data_ptr<int64_t>(), tokens.stride(0), static_cast<int>(P),
      tokens.size(1), tok_in.data_ptr<int64_t>(), reinterpret_cast<long long*>(rng.data_ptr<int64_t>()),
      lp.has_value() ? lp->data_ptr<float>() : nullptr, lp.has_value() ? lp_all->data_ptr<float>() : nullptr,
      lp.has_value() ? lp_all->stride(0) : 0, lp.has_value() ? lp_all->size(1) : 0,
      device_status_ptr(nxt.get_device()));
  TT_CUDA_CHECK(cudaGetLastError());
}

// tokens int64 [B]; logprob fp32 [B] (optional).  top_k <= 0: off; top_p outside (0, 1): off.
// rng (optional, int64 [2] on the device): seed and offset read by the kernel instead of the
// host values, so a captured graph draws a new number on every replay.
void sample_tokens(torch::Tensor logits, double temperature, int64_t top_k, double top_p, int64_t seed,
                   int64_t offset, torch::Tensor tokens, c10::optional<torch::Tensor> logprob,
                   c10::optional<torch::Tensor> rng) {
  TT_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "sample: logits must be CUDA [B, V]");
  TT_CHECK(temperature > 0, "sample: temperature must be > 0");
  TT_CHECK(tokens.scalar_type() == torch::kInt64 && tokens.numel() == logits.size(0) && tokens.is_contiguous(),
           "sample: tokens int64 [B]");
  float* lp = nullptr;
  if (logprob.has_value()) {
    TT_CHECK(logprob->scalar_type() == torch::kFloat32 && logprob->numel() == logits.size(0), "sample: logprob [B]");
    lp = logprob->data_ptr<float>();
  }
  const long long* rng_p = nullptr;
  if (rng.has_value()) {
    TT_CHECK(rng->is_cuda() && rng->scalar_type() == torch::kInt64 && rng->numel() >= 2, "sample: rng int64 [2]");
    rng_p = reinterpret_cast<const long long*>(rng->data_ptr<int64_t>());
  }
  const int64_t B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  const float inv_t = static_cast<float>(1.0 / temperature);
  const int k = static_cast<int>(top_k > 0 ? std::min<int64_t>(top_k, V) : 0);
  if (logits.scalar_type() == torch::kBFloat16) {
    sample::sample_kernel<__nv_bfloat16><<<static_cast<unsigned>(B), sample::THREADS, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), static_cast<int>(V), logits.stride(0), inv_t, k,
        static_cast<float>(top_p), static_cast<unsigned long long>(seed), static_cast<unsigned long long>(offset),
        rng_p, tokens.data_ptr<int64_t>(), lp);
  } else {
    TT_CHECK(logits.scalar_type() == torch::kFloat32, "sample: logits bf16 or fp32");
    sample::sample_kernel<float><<<static_cast<unsigned>(B), sample::THREADS, 0, cur_stream()>>>(
        logits.data_ptr<float>(), static_cast<int>(V), logits.stride(0), inv_t, k, static_cast<float>(top_p),
        static_cast<unsigned long long>(seed), static_cast<unsigned long long>(offset), rng_p, tokens.data_ptr<int64_t>(),
        lp);
  }
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
