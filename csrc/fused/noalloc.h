// Allocation-free entry point for the fused residual-add + RMSNorm kernel.
//
// This entry point has no counterpart in the reference library. It exists for
// callers that are not allowed to allocate device memory when they run: for
// example a plugin invoked by an inference engine that owns every byte of GPU
// memory and forbids cudaMalloc after start-up, or code that runs while the
// process's allocator is disabled. Those callers pass inputs and outputs only;
// the kernel's scratch space (its signal block and staging slots) lives in a
// fixed-size array compiled into the library.
//
// Limits and rules:
//  * one rank (no cross-GPU reduction): y = RMSNorm(x + residual) * gamma and
//    residual_out = x + residual, bf16, row-major [rows, hidden];
//  * rows * hidden * 2 bytes must not exceed B200AR_NOALLOC_MAX_BYTES (2 MiB),
//    hidden a multiple of 8 and at most 16384; larger requests are rejected;
//  * the scratch array (b200ar_noalloc_scratch_bytes() per GPU: a 16.3 KiB
//    signal block plus two slots of B200AR_NOALLOC_MAX_BYTES) stays resident
//    on every GPU that loads the library until the process exits;
//  * the first call on a device sets up that device (looks up the array's
//    device address and clears its signal block); make that first call before
//    any stream capture;
//  * all calls share the one array, so calls whose executions overlap on the
//    GPU (different streams without ordering, several threads) race and give
//    wrong results: order them on one stream.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define B200AR_NOALLOC_MAX_BYTES (2u << 20)

#ifdef __cplusplus
extern "C" {
#endif

// Returns 0 on success; otherwise a non-zero code whose text is returned by
// b200ar_noalloc_last_error().
__attribute__((visibility("default"))) int b200ar_residual_rmsnorm_noalloc(
    const void* x, const void* residual, const void* gamma, void* y, void* residual_out, int64_t rows,
    int64_t hidden, float eps, cudaStream_t stream);

__attribute__((visibility("default"))) const char* b200ar_noalloc_last_error(void);

// Bytes of the library-resident scratch array on each GPU.
__attribute__((visibility("default"))) int64_t b200ar_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif
