// Fused residual-add + RMSNorm (forward and backward), fp32 residual stream.
//
// Reference semantics (tinytron/model/modules/norm.py:14-19 and the residual adds in
// gpt.py:39-41): the residual x is fp32, y = w * (x * rsqrt(mean(x^2) + eps)) with
// fp32 math; the result feeds a bf16 projection, so it is emitted directly as bf16.
//
// forward:  x_out = x + delta (delta optional, bf16);  h = bf16(w * x_out * rstd);  rstd saved.
// backward: g = g_x_out + rstd * (w*gh - xhat * mean(w*gh*xhat));   gx = g (fp32),
//           g_delta = bf16(g);  dw partial sums per row-group, reduced deterministically.
#include "common/host_utils.h"
#include "common/ptx.cuh"
#include "fused/rmsnorm_bwd_noalloc.h"

namespace tt {
namespace {

constexpr int EPT = 8;  // elements per thread (one 32-byte fp32 chunk / 16-byte bf16 chunk)

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ void load8_f32(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8_f32(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y), c = unpack_bf16x2(q.z), d = unpack_bf16x2(q.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ void store8_bf16(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                            pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// One CTA per row; blockDim = ceil(D/8 / 32) * 32 threads, thread t owns columns [8t, 8t+8).
__global__ void add_rmsnorm_fwd_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
                                       const float* __restrict__ w, float* __restrict__ x_out,
                                       __nv_bfloat16* __restrict__ h, float* __restrict__ rstd_out, int D,
                                       float eps) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int c = threadIdx.x * EPT;
  const bool active = c < D;
  const size_t off = static_cast<size_t>(row) * D + c;
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float ss = 0.0f;
  if (active) {
    load8_f32(x + off, v);
    if (delta != nullptr) {
      float d[8];
      load8_bf16(delta + off, d);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] += d[i];
    }
    if (x_out != nullptr) store8_f32(x_out + off, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
  const float tot = block_sum(ss, red);
  const float r = rsqrtf(tot / static_cast<float>(D) + eps);
  if (threadIdx.x == 0 && rstd_out != nullptr) rstd_out[row] = r;
  if (active) {
    float wv[8], o[8];
    load8_f32(w + c, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = wv[i] * (v[i] * r);
    store8_bf16(h + off, o);
  }
}

// ROWS rows per CTA so dw partials are per CTA (deterministic two-stage reduction).
constexpr int BWD_ROWS = 16;

__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ gh, const float* __restrict__ x,
                                   const float* __restrict__ rstd, const float* __restrict__ w,
                                   const float* __restrict__ g_res, float* __restrict__ gx,
                                   __nv_bfloat16* __restrict__ g_delta, float* __restrict__ dw_part, int M, int D) {
  __shared__ float red[32];
  const int c = threadIdx.x * EPT;
  const bool active = c < D;
  float wv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float dw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (active) load8_f32(w + c, wv);
  const int row0 = blockIdx.x * BWD_ROWS;
  for (int rr = 0; rr < BWD_ROWS; ++rr) {
    const int row = row0 + rr;
    if (row >= M) break;  // uniform across the CTA
    const size_t off = static_cast<size_t>(row) * D + c;
    const float r = rstd[row];
    float xv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float dot = 0.0f;
    if (active) {
      load8_f32(x + off, xv);
      load8_bf16(gh + off, g);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = xv[i] * r;
        dw[i] += g[i] * xh;
        g[i] *= wv[i];
        dot += g[i] * xh;
        xv[i] = xh;
      }
    }
    const float mean_dot = block_sum(dot, red) / static_cast<float>(D);
    if (active) {
      float o[8];
      float res[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (g_res != nullptr) load8_f32(g_res + off, res);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = res[i] + r * (g[i] - xv[i] * mean_dot);
      if (gx != nullptr) store8_f32(gx + off, o);
      if (g_delta != nullptr) store8_bf16(g_delta + off, o);
    }
  }
  if (active && dw_part != nullptr) store8_f32(dw_part + static_cast<size_t>(blockIdx.x) * D + c, dw);
}

// dw[d] (+)= sum_g part[g, d]   (fixed summation order -> deterministic).
// Block = 32 columns x 8 row lanes (256 threads): row lane r sums rows g = r (mod 8) with
// four independent accumulators, then the 8 lane sums are added in lane order.
constexpr int RR_COLS = 32;
__global__ void __launch_bounds__(256) reduce_rows_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                          int G, int D, int accumulate) {
  __shared__ float red[8][RR_COLS + 1];
  const int cx = threadIdx.x & 31, ry = threadIdx.x >> 5;
  const int d = blockIdx.x * RR_COLS + cx;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (d < D) {
    int g = ry;
    for (; g + 24 < G; g += 32) {
      s0 += part[static_cast<size_t>(g) * D + d];
      s1 += part[static_cast<size_t>(g + 8) * D + d];
      s2 += part[static_cast<size_t>(g + 16) * D + d];
      s3 += part[static_cast<size_t>(g + 24) * D + d];
    }
    for (; g < G; g += 8) s0 += part[static_cast<size_t>(g) * D + d];
  }
  red[ry][cx] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (ry == 0 && d < D) {
    float s = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) s += red[r][cx];
    out[d] = accumulate ? out[d] + s : s;
  }
}

int norm_threads(int D) { return ((D / EPT + 31) / 32) * 32; }

}  // namespace

// x: [M, D] fp32; delta: [M, D] bf16 or None; w: [D] fp32.
// Writes x_out (may be None) fp32, h bf16, rstd [M] fp32.
void add_rmsnorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> delta, torch::Tensor w,
                     c10::optional<torch::Tensor> x_out, torch::Tensor h, torch::Tensor rstd, double eps) {
  TT_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "x must be contiguous fp32 CUDA");
  const int64_t D = x.size(-1);
  const int64_t M = x.numel() / D;
  TT_CHECK(D % EPT == 0 && D / EPT <= 1024, "hidden size must be a multiple of 8 and <= 8192");
  TT_CHECK(w.scalar_type() == torch::kFloat32 && w.numel() == D, "w must be fp32 [D]");
  check_cuda_bf16(h, "h");
  TT_CHECK(h.is_contiguous() && h.numel() == M * D, "h shape");
  TT_CHECK(rstd.scalar_type() == torch::kFloat32 && rstd.numel() == M, "rstd must be fp32 [M]");
  const __nv_bfloat16* dp = nullptr;
  if (delta.has_value()) {
    check_cuda_bf16(*delta, "delta");
    TT_CHECK(delta->is_contiguous() && delta->numel() == M * D, "delta shape");
    dp = reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr());
  }
  float* xo = nullptr;
  if (x_out.has_value()) {
    TT_CHECK(x_out->scalar_type() == torch::kFloat32 && x_out->is_contiguous() && x_out->numel() == M * D,
             "x_out shape");
    xo = x_out->data_ptr<float>();
  }
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  add_rmsnorm_fwd_kernel<<<static_cast<unsigned>(M), norm_threads(static_cast<int>(D)), 0, cur_stream()>>>(
      x.data_ptr<float>(), dp, w.data_ptr<float>(), xo, reinterpret_cast<__nv_bfloat16*>(h.data_ptr()),
      rstd.data_ptr<float>(), static_cast<int>(D), static_cast<float>(eps));
  TT_CUDA_CHECK(cudaGetLastError());
}

// gh: [M, D] bf16 grad of h; x: [M, D] fp32 (the normalised input, i.e. x_out of fwd);
// rstd [M]; w [D]; g_res: [M, D] fp32 grad flowing into x_out from the residual path (or None).
// Writes gx fp32 (may be None), g_delta bf16 (may be None), and dw (+)= into dw [D] fp32.
void rmsnorm_bwd(torch::Tensor gh, torch::Tensor x, torch::Tensor rstd, torch::Tensor w,
                 c10::optional<torch::Tensor> g_res, c10::optional<torch::Tensor> gx,
                 c10::optional<torch::Tensor> g_delta, torch::Tensor dw, bool accumulate_dw, torch::Tensor scratch) {
  check_cuda_bf16(gh, "gh");
  const int64_t D = x.size(-1);
  const int64_t M = x.numel() / D;
  TT_CHECK(D % EPT == 0 && D / EPT <= 1024, "hidden size must be a multiple of 8 and <= 8192");
  TT_CHECK(gh.is_contiguous() && gh.numel() == M * D && x.is_contiguous(), "rmsnorm_bwd shapes");
  TT_CHECK(dw.scalar_type() == torch::kFloat32 && dw.numel() == D, "dw must be fp32 [D]");
  const int G = static_cast<int>((M + BWD_ROWS - 1) / BWD_ROWS);
  TT_CHECK(scratch.scalar_type() == torch::kFloat32 && scratch.numel() >= static_cast<int64_t>(G) * D,
           "scratch too small");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = cur_stream();
  const float* gr = g_res.has_value() ? g_res->data_ptr<float>() : nullptr;
  float* gxp = gx.has_value() ? gx->data_ptr<float>() : nullptr;
  __nv_bfloat16* gdp = g_delta.has_value() ? reinterpret_cast<__nv_bfloat16*>(g_delta->data_ptr()) : nullptr;
  rmsnorm_bwd_kernel<<<G, norm_threads(static_cast<int>(D)), 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(gh.data_ptr()), x.data_ptr<float>(), rstd.data_ptr<float>(),
      w.data_ptr<float>(), gr, gxp, gdp, scratch.data_ptr<float>(), static_cast<int>(M), static_cast<int>(D));
  TT_CUDA_CHECK(cudaGetLastError());
  reduce_rows_kernel<<<static_cast<unsigned>((D + RR_COLS - 1) / RR_COLS), 256, 0, st>>>(
      scratch.data_ptr<float>(), dw.data_ptr<float>(), G, static_cast<int>(D), accumulate_dw ? 1 : 0);
  TT_CUDA_CHECK(cudaGetLastError());
}

int64_t rmsnorm_bwd_scratch_numel(int64_t M, int64_t D) { return ((M + BWD_ROWS - 1) / BWD_ROWS) * D; }

}  // namespace tt

// ----------------------------------------------------------------------------------------------
// Allocation-free variant of rmsnorm_bwd (see fused/rmsnorm_bwd_noalloc.h). Same kernels; the
// weight-gradient partials live in a file-scope device array instead of a caller-provided
// buffer. Host code must not hand the array's name to a kernel (on the host it is only a
// stand-in for the symbol): its device address is looked up once per device below.
static __device__ __align__(256) float tt_rmsnorm_noalloc_scratch[TT_RMSNORM_NOALLOC_MAX_SCRATCH];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {nullptr};

float* noalloc_scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = 3;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, tt_rmsnorm_noalloc_scratch) != cudaSuccess || p == nullptr) {
      *err = 3;
      return nullptr;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  return g_noalloc_ptr[dev];
}
}  // namespace

extern "C" __attribute__((visibility("default"))) int tt_rmsnorm_bwd_noalloc(
    const __nv_bfloat16* gh, const float* x, const float* rstd, const float* w, const float* g_res, float* gx,
    __nv_bfloat16* g_delta, float* dw, int M, int D, int accumulate_dw, cudaStream_t stream) {
  using namespace tt;
  // An error left pending on this thread by earlier, unrelated work would otherwise be
  // picked up (and cleared) by the launch checks below and reported as this call's launch
  // failure; report it as such instead and launch nothing.
  if (cudaPeekAtLastError() != cudaSuccess) return 5;
  if (gh == nullptr || x == nullptr || rstd == nullptr || w == nullptr || dw == nullptr || M < 0 || D <= 0 ||
      D % EPT != 0 || D / EPT > 1024)
    return 1;
  if (M == 0) return 0;
  const long long G = (static_cast<long long>(M) + BWD_ROWS - 1) / BWD_ROWS;
  if (G * D > TT_RMSNORM_NOALLOC_MAX_SCRATCH) return 2;
  int err = 0;
  float* scratch = noalloc_scratch_for_current_device(&err);
  if (scratch == nullptr) return err ? err : 3;
  rmsnorm_bwd_kernel<<<static_cast<unsigned>(G), norm_threads(D), 0, stream>>>(gh, x, rstd, w, g_res, gx, g_delta,
                                                                            scratch, M, D);
  if (cudaGetLastError() != cudaSuccess) return 4;
  reduce_rows_kernel<<<static_cast<unsigned>((D + RR_COLS - 1) / RR_COLS), 256, 0, stream>>>(scratch, dw, static_cast<int>(G), D,
                                                                                accumulate_dw ? 1 : 0);
  if (cudaGetLastError() != cudaSuccess) return 4;
  return 0;
}

