// Host-side helpers shared by the CUDA extension: tensor-map encoding (driver entry
// point fetched through the runtime, so nothing links against libcuda directly),
// device properties and argument checks.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <stdexcept>
#include <string>

#define TT_CHECK(cond, msg)                                                     \
  do {                                                                          \
    if (!(cond)) throw std::runtime_error(std::string("tinytron_b200: ") + msg); \
  } while (0)

#define TT_CUDA_CHECK(expr)                                                                 \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    if (_e != cudaSuccess)                                                                  \
      throw std::runtime_error(std::string("tinytron_b200 CUDA error: ") + cudaGetErrorString(_e) + \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__));         \
  } while (0)

namespace tt {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    TT_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TT_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled entry point not found");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [outer, inner] with the given row
// stride (bytes), 128-byte swizzle, box {box_inner, box_outer}.  Out-of-range
// elements of a box read as zero.
inline CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                                     uint32_t box_inner, uint32_t box_outer,
                                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  TT_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  TT_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return m;
}

// 2-D fp32 tensor map over a row-major matrix [outer, inner] (row stride in bytes),
// box {box_inner, box_outer}; used as the destination of TMA reductions.
inline CUtensorMap make_tmap_2d_f32(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                                    uint32_t box_inner, uint32_t box_outer,
                                    CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  TT_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  TT_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return m;
}

inline int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 64 && cached[device]) return cached[device];
  int n = 0;
  TT_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  if (device < 64) cached[device] = n;
  return n;
}

inline cudaStream_t cur_stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

inline void check_cuda_bf16(const torch::Tensor& t, const char* name) {
  TT_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  TT_CHECK(t.scalar_type() == torch::kBFloat16, std::string(name) + " must be bfloat16");
}

// Per-device status word for bounded device-side waits (see ptx.cuh).
int* device_status_ptr(int device);

}  // namespace tt
