// Memory-bound kernels of the training step:
//   * RoPE (HF half-split rotation) applied in place on the packed q|k|v buffer
//     (reference: tinytron/model/modules/attn.py:13-63); backward = inverse rotation.
//   * Cross-entropy over bf16 logits with ignore_index: per-row loss + LSE, and the
//     unscaled gradient softmax - onehot written in place over the logits
//     (reference: tinytron/model/modules/loss.py:19-43).
//   * Embedding gather (fp32 table -> fp32 residual) and its scatter-add backward
//     into the fp32 master grad (reference: gpt.py:94).
//   * Fused AdamW over flat fp32 buffers that also refreshes the bf16 weight shadow
//     and applies the grad-clip coefficient read from device memory
//     (torch.optim.AdamW math, used by the reference in trainer.py:227-234).
//   * Sum of squares / clip coefficient for global-norm clipping (gpt.py:143-163).
#include "common/host_utils.h"
#include "common/ptx.cuh"
#include "common/fast_exp2.cuh"

namespace tt {
namespace {

// ----------------------------------------------------------------- RoPE
// One thread rotates 8 pairs (j, j+d/2) of one (row, head).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, int ld, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, int M, int T, int pos_offset, int n_heads, int d,
                            float sign) {
  const int half = d >> 1;
  const int groups = half >> 3;  // threads per head
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(M) * n_heads * groups;
  if (idx >= total) return;
  const int gi = static_cast<int>(idx % groups);
  const long long rh = idx / groups;
  const int head = static_cast<int>(rh % n_heads);
  const int row = static_cast<int>(rh / n_heads);
  const int pos = row % T + pos_offset;
  const int j0 = gi * 8;
  __nv_bfloat16* base = qkv + static_cast<size_t>(row) * ld + static_cast<size_t>(head) * d;
  uint4 lo = *reinterpret_cast<const uint4*>(base + j0);
  uint4 hi = *reinterpret_cast<const uint4*>(base + half + j0);
  const float4* cp = reinterpret_cast<const float4*>(cos_t + static_cast<size_t>(pos) * half + j0);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + static_cast<size_t>(pos) * half + j0);
  const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
  const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  uint32_t* lw = reinterpret_cast<uint32_t*>(&lo);
  uint32_t* hw = reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = unpack_bf16x2(lw[i]);
    const float2 b = unpack_bf16x2(hw[i]);
    const float ca = cs[2 * i], cb = cs[2 * i + 1];
    const float sa = sign * sn[2 * i], sb = sign * sn[2 * i + 1];
    // out_lo = x_lo*cos - x_hi*sin ; out_hi = x_hi*cos + x_lo*sin
    lw[i] = pack_bf16x2(a.x * ca - b.x * sa, a.y * cb - b.y * sb);
    hw[i] = pack_bf16x2(b.x * ca + a.x * sa, b.y * cb + a.y * sb);
  }
  *reinterpret_cast<uint4*>(base + j0) = lo;
  *reinterpret_cast<uint4*>(base + half + j0) = hi;
}

// ----------------------------------------------------------------- cross-entropy
constexpr int CE_THREADS = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * __expf(m - m2) + s2;
    m = m2;
  } else if (m2 != -INFINITY) {
    s += s2 * __expf(m2 - m);
  }
}

__global__ void __launch_bounds__(CE_THREADS) ce_fwd_kernel(__nv_bfloat16* __restrict__ logits, int ld,
                                                            const int64_t* __restrict__ targets,
                                                            float* __restrict__ loss, float* __restrict__ lse_out,
                                                            int V, int ignore_index, int write_grad) {
  __shared__ float sm_m[CE_THREADS / 32], sm_s[CE_THREADS / 32];
  const int row = blockIdx.x;
  __nv_bfloat16* x = logits + static_cast<size_t>(row) * ld;
  const int64_t tgt = targets[row];
  const bool valid = tgt != ignore_index;
  float m = -INFINITY, s = 0.0f;
  const int nvec = V / 8;
  for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
    const uint4 q = reinterpret_cast<const uint4*>(x)[i];
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&q);
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16x2(w[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
    float lm = v[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) lm = fmaxf(lm, v[k]);
    float ls = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ls += __expf(v[k] - lm);
    online_merge(m, s, lm, ls);
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += CE_THREADS) online_merge(m, s, __bfloat162float(x[i]), 1.0f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[warp] = m;
    sm_s[warp] = s;
  }
  __syncthreads();
  m = sm_m[0];
  s = sm_s[0];
  for (int wi = 1; wi < CE_THREADS / 32; ++wi) online_merge(m, s, sm_m[wi], sm_s[wi]);
  const float lse = m + __logf(s);
  if (threadIdx.x == 0) {
    if (lse_out != nullptr) lse_out[row] = lse;
    loss[row] = valid ? (lse - __bfloat162float(x[tgt])) : 0.0f;
  }
  if (!write_grad) return;
  __syncthreads();  // every thread has read x[tgt] / its chunk before it is overwritten
  for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
    uint4 q = reinterpret_cast<uint4*>(x)[i];
    uint32_t* w = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16x2(w[k]);
      const int c = i * 8 + 2 * k;
      float g0 = valid ? __expf(f.x - lse) - (c == tgt ? 1.0f : 0.0f) : 0.0f;
      float g1 = valid ? __expf(f.y - lse) - (c + 1 == tgt ? 1.0f : 0.0f) : 0.0f;
      w[k] = pack_bf16x2(g0, g1);
    }
    reinterpret_cast<uint4*>(x)[i] = q;
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += CE_THREADS) {
    const float f = __bfloat162float(x[i]);
    x[i] = __float2bfloat16_rn(valid ? __expf(f - lse) - (i == tgt ? 1.0f : 0.0f) : 0.0f);
  }
}

// ----------------------------------------------------------------- embedding
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ table,
                                     float* __restrict__ out, int D) {
  const int row = blockIdx.x;
  const int64_t t = idx[row];
  const float4* src = reinterpret_cast<const float4*>(table + static_cast<size_t>(t) * D);
  float4* dst = reinterpret_cast<float4*>(out + static_cast<size_t>(row) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = src[i];
}

// Embedding backward: token ids sorted (stable) beforehand; the block at the first
// position of each run of equal ids sums that run's gradient rows in position order and
// adds the sum into the table row once (no atomics, fixed summation order).
__global__ void embedding_bwd_sorted_kernel(const int64_t* __restrict__ sorted_idx, const int64_t* __restrict__ order,
                                            int N, const float* __restrict__ g, float* __restrict__ gtable, int D,
                                            long long V, int* status) {
  const int pos = blockIdx.x;
  const int64_t t = sorted_idx[pos];
  if (pos > 0 && sorted_idx[pos - 1] == t) return;  // not the first of its run
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0) atomicCAS(status, 0, static_cast<int>(kBadIndex));
    return;
  }
  int end = pos + 1;
  while (end < N && sorted_idx[end] == t) ++end;
  float4* dst = reinterpret_cast<float4*>(gtable + static_cast<size_t>(t) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) {
    float4 acc = dst[i];
    for (int j = pos; j < end; ++j) {
      const float4 v = reinterpret_cast<const float4*>(g + static_cast<size_t>(order[j]) * D)[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    dst[i] = acc;
  }
}

// ----------------------------------------------------------------- AdamW
struct AdamArgs {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt;
  const float* grad_scale;  // optional device scalar (clip coefficient)
};

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ p16, long long n, AdamArgs a) {
  const float gs = a.grad_scale != nullptr ? *a.grad_scale : 1.0f;
  const float step = a.lr / a.bc1;
  const float decay = 1.0f - a.lr * a.wd;
  const long long n4 = n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    float4 gv = reinterpret_cast<const float4*>(g)[i];
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = &pv.x;
    float* gp = &gv.x;
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
    reinterpret_cast<float4*>(p)[i] = pv;
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p16 != nullptr) {
      uint2 o;
      o.x = pack_bf16x2(pv.x, pv.y);
      o.y = pack_bf16x2(pv.z, pv.w);
      reinterpret_cast<uint2*>(p16)[i] = o;
    }
  }
  // tail
  for (long long i = n4 * 4 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gr = g[i] * gs;
    float pv = p[i] * decay;
    m[i] = m[i] + (1.0f - a.beta1) * (gr - m[i]);
    v[i] = a.beta2 * v[i] + (1.0f - a.beta2) * gr * gr;
    pv -= step * (m[i] / (sqrtf(v[i]) / a.bc2_sqrt + a.eps));
    p[i] = pv;
    if (p16 != nullptr) p16[i] = __float2bfloat16_rn(pv);
  }
}

// ----------------------------------------------------------------- sum of squares
constexpr int SS_THREADS = 512;

__global__ void sumsq_kernel(const float* __restrict__ x, long long n, float* __restrict__ partial) {
  __shared__ float red[SS_THREADS / 32];
  float s = 0.0f;
  const long long n4 = n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long long i = n4 * 4 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    s += x[i] * x[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < SS_THREADS / 32; ++i) t += red[i];
    partial[blockIdx.x] = t;
  }
}

// out[0] (+)= sum(partial[0..G)) in a fixed order.
__global__ void sum_partials_kernel(const float* __restrict__ partial, int G, float* __restrict__ out, int accumulate) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < G; i += blockDim.x) s += partial[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) t += red[i];
    out[0] = accumulate ? out[0] + static_cast<float>(t) : static_cast<float>(t);
  }
}

// norm = sqrt(sumsq); coef = min(max_norm / (norm + 1e-6), 1)
__global__ void clip_coef_kernel(const float* __restrict__ sumsq, float* __restrict__ norm_out,
                                 float* __restrict__ coef_out, float max_norm) {
  const float nrm = sqrtf(sumsq[0]);
  norm_out[0] = nrm;
  coef_out[0] = fminf(max_norm / (nrm + 1e-6f), 1.0f);
}

__global__ void exp2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = exp2_poly(x[i]);
}

}  // namespace

// Elementwise 2^x with the FMA-pipe polynomial used inside the attention kernels (for testing).
void exp2_poly_op(torch::Tensor x, torch::Tensor y) {
  TT_CHECK(x.scalar_type() == torch::kFloat32 && y.scalar_type() == torch::kFloat32 && x.is_contiguous() &&
               y.is_contiguous() && x.numel() == y.numel(),
           "exp2_poly: fp32 contiguous tensors of equal size");
  const long long n = x.numel();
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  exp2_poly_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, cur_stream()>>>(x.data_ptr<float>(),
                                                                                   y.data_ptr<float>(), n);
  TT_CUDA_CHECK(cudaGetLastError());
}

void rope_inplace(torch::Tensor qkv, torch::Tensor cos_t, torch::Tensor sin_t, int64_t T, int64_t pos_offset,
                  int64_t n_heads, int64_t head_dim, bool inverse) {
  check_cuda_bf16(qkv, "qkv");
  TT_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.stride(0) % 8 == 0, "qkv must be 2-D row-major");
  TT_CHECK(head_dim % 16 == 0, "head_dim must be a multiple of 16");
  TT_CHECK(n_heads * head_dim <= qkv.size(1), "qkv too narrow");
  const int64_t M = qkv.size(0);
  TT_CHECK(cos_t.scalar_type() == torch::kFloat32 && sin_t.scalar_type() == torch::kFloat32 &&
               cos_t.size(1) == head_dim / 2,
           "cos/sin tables must be fp32 [max_pos, d/2]");
  TT_CHECK((T - 1) + pos_offset < cos_t.size(0) && pos_offset >= 0, "position beyond rope table");
  if (M == 0 || n_heads == 0) return;
  const c10::cuda::CUDAGuard guard(qkv.device());
  const long long total = M * n_heads * (head_dim / 16);
  const int threads = 256;
  rope_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), static_cast<int>(qkv.stride(0)), cos_t.data_ptr<float>(),
      sin_t.data_ptr<float>(), static_cast<int>(M), static_cast<int>(T), static_cast<int>(pos_offset),
      static_cast<int>(n_heads), static_cast<int>(head_dim), inverse ? -1.0f : 1.0f);
  TT_CUDA_CHECK(cudaGetLastError());
}

void cross_entropy_fwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss,
                       c10::optional<torch::Tensor> lse, int64_t ignore_index, bool write_grad) {
  check_cuda_bf16(logits, "logits");
  TT_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.stride(0) % 8 == 0, "logits must be [M, V]");
  TT_CHECK(targets.scalar_type() == torch::kInt64 && targets.numel() == logits.size(0), "targets must be int64 [M]");
  TT_CHECK(loss.scalar_type() == torch::kFloat32 && loss.numel() == logits.size(0), "loss must be fp32 [M]");
  const int64_t M = logits.size(0);
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  ce_fwd_kernel<<<static_cast<unsigned>(M), CE_THREADS, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), static_cast<int>(logits.stride(0)),
      targets.data_ptr<int64_t>(), loss.data_ptr<float>(), lse.has_value() ? lse->data_ptr<float>() : nullptr,
      static_cast<int>(logits.size(1)), static_cast<int>(ignore_index), write_grad ? 1 : 0);
  TT_CUDA_CHECK(cudaGetLastError());
}

void embedding_fwd(torch::Tensor idx, torch::Tensor table, torch::Tensor out) {
  TT_CHECK(idx.scalar_type() == torch::kInt64 && table.scalar_type() == torch::kFloat32 &&
               out.scalar_type() == torch::kFloat32,
           "embedding dtypes");
  const int64_t D = table.size(1);
  TT_CHECK(D % 4 == 0 && out.numel() == idx.numel() * D && table.is_contiguous() && out.is_contiguous(),
           "embedding shapes");
  if (idx.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(table.device());
  embedding_fwd_kernel<<<static_cast<unsigned>(idx.numel()), 256, 0, cur_stream()>>>(
      idx.data_ptr<int64_t>(), table.data_ptr<float>(), out.data_ptr<float>(), static_cast<int>(D));
  TT_CUDA_CHECK(cudaGetLastError());
}

void embedding_bwd(torch::Tensor idx, torch::Tensor g, torch::Tensor gtable) {
  const int64_t D = gtable.size(1);
  TT_CHECK(g.scalar_type() == torch::kFloat32 && gtable.scalar_type() == torch::kFloat32 && g.is_contiguous() &&
               gtable.is_contiguous() && D % 4 == 0,
           "embedding_bwd dtypes/shapes");
  if (idx.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(g.device());
  // Stable sort of the token ids (device radix sort), then one pass over the runs:
  // deterministic, unlike per-token atomic adds.
  auto flat = idx.reshape({-1}).contiguous();
  auto sr = flat.sort(/*stable=*/true, /*dim=*/0, /*descending=*/false);
  auto sorted = std::get<0>(sr);
  auto order = std::get<1>(sr);
  embedding_bwd_sorted_kernel<<<static_cast<unsigned>(flat.numel()), 256, 0, cur_stream()>>>(
      sorted.data_ptr<int64_t>(), order.data_ptr<int64_t>(), static_cast<int>(flat.numel()), g.data_ptr<float>(),
      gtable.data_ptr<float>(), static_cast<int>(D), gtable.size(0), device_status_ptr(g.get_device()));
  TT_CUDA_CHECK(cudaGetLastError());
}

void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p16,
                double lr, double beta1, double beta2, double eps, double wd, int64_t step,
                c10::optional<torch::Tensor> grad_scale) {
  TT_CHECK(p.scalar_type() == torch::kFloat32 && g.scalar_type() == torch::kFloat32 &&
               m.scalar_type() == torch::kFloat32 && v.scalar_type() == torch::kFloat32,
           "adamw: fp32 buffers expected");
  const int64_t n = p.numel();
  TT_CHECK(g.numel() == n && m.numel() == n && v.numel() == n && p.is_contiguous() && g.is_contiguous() &&
               m.is_contiguous() && v.is_contiguous(),
           "adamw: shapes");
  for (auto* t : {&p, &g, &m, &v})
    TT_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "adamw: buffers must be 16-byte aligned");
  __nv_bfloat16* p16p = nullptr;
  if (p16.has_value()) {
    check_cuda_bf16(*p16, "p16");
    TT_CHECK(p16->numel() == n && p16->is_contiguous() && reinterpret_cast<uintptr_t>(p16->data_ptr()) % 8 == 0,
             "adamw: p16 shape/alignment");
    p16p = reinterpret_cast<__nv_bfloat16*>(p16->data_ptr());
  }
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(p.device());
  AdamArgs a;
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  a.grad_scale = nullptr;
  if (grad_scale.has_value()) a.grad_scale = grad_scale->data_ptr<float>();
  const int sms = num_sms(p.get_device());
  const long long want = (n / 4 + 255) / 256;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>(want, sms * 8)));
  adamw_kernel<<<grid, 256, 0, cur_stream()>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                               v.data_ptr<float>(), p16p, n, a);
  TT_CUDA_CHECK(cudaGetLastError());
}

// out[0] (+)= sum(x^2); scratch needs >= 8 * num_SMs floats.
void sumsq(torch::Tensor x, torch::Tensor out, torch::Tensor scratch, bool accumulate) {
  TT_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && out.scalar_type() == torch::kFloat32,
           "sumsq: fp32 contiguous expected");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t n = x.numel();
  const int sms = num_sms(x.get_device());
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((n / 4 + SS_THREADS - 1) / SS_THREADS, sms * 8)));
  TT_CHECK(scratch.numel() >= grid && scratch.scalar_type() == torch::kFloat32, "sumsq: scratch too small");
  cudaStream_t st = cur_stream();
  if (n > 0) {
    TT_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "sumsq: 16-byte alignment");
    sumsq_kernel<<<grid, SS_THREADS, 0, st>>>(x.data_ptr<float>(), n, scratch.data_ptr<float>());
    TT_CUDA_CHECK(cudaGetLastError());
    sum_partials_kernel<<<1, 1024, 0, st>>>(scratch.data_ptr<float>(), grid, out.data_ptr<float>(), accumulate ? 1 : 0);
  } else if (!accumulate) {
    out.zero_();
  }
  TT_CUDA_CHECK(cudaGetLastError());
}

void clip_coef(torch::Tensor sumsq_t, torch::Tensor norm_out, torch::Tensor coef_out, double max_norm) {
  const c10::cuda::CUDAGuard guard(sumsq_t.device());
  clip_coef_kernel<<<1, 1, 0, cur_stream()>>>(sumsq_t.data_ptr<float>(), norm_out.data_ptr<float>(),
                                              coef_out.data_ptr<float>(), static_cast<float>(max_norm));
  TT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace tt
