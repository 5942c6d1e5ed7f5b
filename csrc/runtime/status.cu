// Per-device status word written by bounded device-side waits (see
// csrc/common/ptx.cuh).  Zero means healthy; a nonzero value is the first
// StatusCode recorded by a wait that gave up.  Allocated once per device and
// kept for the life of the process.
#include "common/host_utils.h"

namespace tt {

int* device_status_ptr(int device) {
  static int* ptrs[64] = {nullptr};
  static std::mutex mu;
  TT_CHECK(device >= 0 && device < 64, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[device] == nullptr) {
    int prev = 0;
    TT_CUDA_CHECK(cudaGetDevice(&prev));
    TT_CUDA_CHECK(cudaSetDevice(device));
    TT_CUDA_CHECK(cudaMalloc(&ptrs[device], 64 * sizeof(int)));
    TT_CUDA_CHECK(cudaMemset(ptrs[device], 0, 64 * sizeof(int)));
    TT_CUDA_CHECK(cudaSetDevice(prev));
  }
  return ptrs[device];
}

// Returns the status word (synchronising the device's current stream first).
int64_t status_read(int64_t device) {
  int* p = device_status_ptr(static_cast<int>(device));
  int v = 0;
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  TT_CUDA_CHECK(cudaStreamSynchronize(cur_stream()));
  TT_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

void status_clear(int64_t device) {
  int* p = device_status_ptr(static_cast<int>(device));
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  TT_CUDA_CHECK(cudaMemsetAsync(p, 0, sizeof(int), cur_stream()));
}

}  // namespace tt
