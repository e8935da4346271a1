// Allocation-free entry point of the lora_kernel_b200 CUDA library.
//
// This entry point has no counterpart in the reference (sudish80/Lora-Kernel-).
// It exists for callers that cannot call cudaMalloc: code running inside a
// host that forbids device allocations after start-up (for example a serving
// process whose memory pool is fixed up front, or a plug-in loaded into
// someone else's CUDA context), and C callers that have no allocator at hand
// to provide scratch buffers.
//
// lk_rmsnorm_bwd_noalloc computes exactly what lk_rmsnorm_bwd computes (RMSNorm
// backward: dx, and dgamma summed over rows), but instead of asking the caller
// for an fp32 scratch buffer of per-block dgamma partials it uses one
// file-scope device array of LK_NOALLOC_NORM_SCRATCH_FLOATS floats (4 MiB).
// Every GPU that loads the library holds that array until the process exits.
//
// Rules for callers:
//  * The caller still provides every input and output (dy, x, gamma, rstd,
//    optional dres, dx, dgamma).  Nothing is allocated, and no cudaMalloc,
//    cudaFree or allocating library routine is called.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture on that device.
//  * A call needs min(ceil(M/8), 2 x SM count) x D floats of scratch; larger
//    requests are rejected with return code -1 and a message from
//    lk_last_error() (on a 148-SM B200: any M for D <= 2048, M <= 2048 rows for
//    D = 4096).
//  * All calls share the one array and it keeps the last call's contents.
//    Every partial a call reads is written by that same call first, so nothing
//    needs clearing between calls, but calls that can overlap on the GPU (on
//    different streams, or from several host threads) race on the array:
//    serialise them.
#pragma once

#include <cuda_runtime.h>

#include "lk_api.h"

#define LK_NOALLOC_NORM_SCRATCH_FLOATS (1 << 20)

#ifdef __cplusplus
extern "C" {
#endif

// Same arguments as LkNormBwdDesc minus the scratch fields; returns 0 or -1.
int lk_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* gamma, const float* rstd,
                           const void* dres, void* dx, float* dgamma, int M, int D, int accumulate,
                           cudaStream_t stream);

#ifdef __cplusplus
}
#endif
