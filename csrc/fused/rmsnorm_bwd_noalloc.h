// Allocation-free RMSNorm backward entry point.
//
// This entry point has no counterpart in the Tinytron reference; it exists for
// callers that cannot allocate device memory themselves: code running inside a
// memory-pool-restricted host process, plugins loaded into a framework whose
// allocator they may not call, or C callers without a CUDA allocator of their
// own. It performs the same computation as the library's regular RMSNorm backward
// (tinytron_b200 `rmsnorm_bwd`), but keeps its scratch space (per-row-group
// partial sums for the weight gradient) in a fixed-size array that is part of the
// loaded library, so it never calls cudaMalloc, cudaFree or any allocating
// library routine. The caller provides every input and output buffer.
//
// Limits and behaviour:
//  * Scratch holds TT_RMSNORM_NOALLOC_MAX_SCRATCH floats (4 MiB) on every GPU that
//    loads the library, kept until the process exits. A call needs
//    ceil(M / 16) * D floats of it; larger problems are rejected (return code 2).
//  * The first call on a device looks up the scratch array's device address for
//    that device (cudaGetSymbolAddress with the device current); make that first
//    call before any CUDA stream capture.
//  * The scratch address is taken for the CURRENT device, so `stream` must belong to
//    the current device (a stream of another device makes the launches fail: code 4).
//  * All calls share the one scratch array and it keeps the last call's partial
//    sums. Every partial a call reads is written by the same call first, so no
//    clearing is needed, but calls whose executions overlap on the GPU (different
//    streams, or concurrent host threads) race on it: serialize them.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#define TT_RMSNORM_NOALLOC_MAX_SCRATCH (1 << 20)

#ifdef __cplusplus
extern "C" {
#endif

// gh:      [M, D] bf16, gradient w.r.t. the normalised output h
// x:       [M, D] fp32, the norm's input (the residual stream after the add)
// rstd:    [M]    fp32, 1/sqrt(mean(x^2) + eps) saved by the forward
// w:       [D]    fp32, norm weight
// g_res:   [M, D] fp32 residual gradient added to the result, or NULL
// gx:      [M, D] fp32 output (may be NULL), g_delta: [M, D] bf16 output (may be NULL)
// dw:      [D]    fp32 weight gradient; accumulated into when accumulate_dw != 0
// Returns 0 on success, 1 for invalid arguments, 2 if ceil(M/16)*D exceeds the
// scratch limit, 3 if the scratch address lookup failed, 4 if a launch failed, and
// 5 if a CUDA error was already pending on the calling thread when the call began
// (nothing is launched then, and the pending error is left for its owner to read).
int tt_rmsnorm_bwd_noalloc(const __nv_bfloat16* gh, const float* x, const float* rstd, const float* w,
                           const float* g_res, float* gx, __nv_bfloat16* g_delta, float* dw, int M, int D,
                           int accumulate_dw, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
