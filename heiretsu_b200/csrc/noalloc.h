// Allocation-free entry point of the extension (C ABI).
//
// This entry point has no counterpart in the reference implementation.
//
// hb_cross_entropy_fwd_noalloc computes the same result as the library's
// regular cross-entropy forward (per-row log-sum-exp of bf16 logits and the
// mean loss over rows) without allocating any device memory. It exists for
// callers that cannot call cudaMalloc or any allocating routine: code running
// inside an allocator's out-of-memory or memory-pressure handler (allocating
// there would re-enter the allocator it is serving), and C/C++ host programs
// that own every device allocation themselves and do not let a library make
// its own. The caller passes all inputs and outputs; the per-row loss scratch
// that the regular entry point asks the caller for lives instead in a
// file-scope device array of HB_CE_NOALLOC_MAX_ROWS floats (256 KB), which
// every GPU that loads the library holds until the process exits.
//
// Rules of use:
// * Rows are limited to HB_CE_NOALLOC_MAX_ROWS; larger M is rejected with
//   HB_NOALLOC_ERR_TOO_LARGE and nothing is launched.
// * The first call on a device (with that device current) looks up the
//   array's device address with cudaGetSymbolAddress; make that first call
//   before any stream capture on the device.
// * All calls share the one array, which keeps the previous call's contents;
//   each call overwrites the rows it uses before reading them. Calls that
//   overlap on the GPU (for example on two streams) race on it: order them
//   on one stream or with events.
// * A target outside [0, V) that is not ignore_index is no class: that row's
//   loss is NaN, so *loss_mean is NaN (this entry point has no status word).
// * M == 0 returns HB_NOALLOC_OK, launches nothing and leaves lse and
//   *loss_mean untouched (they keep whatever the caller put there).
// * Kernels are enqueued on `stream`; the call returns without synchronising.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define HB_CE_NOALLOC_MAX_ROWS 65536

#define HB_NOALLOC_OK 0
#define HB_NOALLOC_ERR_ARG 1        // null pointer, bad V / ld / M, logits not 16-byte aligned
#define HB_NOALLOC_ERR_TOO_LARGE 2  // M > HB_CE_NOALLOC_MAX_ROWS
#define HB_NOALLOC_ERR_CUDA 3       // a CUDA runtime call failed

#ifdef __cplusplus
extern "C" {
#endif

// logits: bf16 [M, ld] (row stride ld elements, ld % 8 == 0, ld >= V), device memory, 16-byte aligned
// targets: int64 [M] class ids (ignore_index rows contribute no loss), device memory
// lse: fp32 [M] output, device memory; loss_mean: fp32 [1] output, device memory
int hb_cross_entropy_fwd_noalloc(const void* logits, long ld, int M, int V, const int64_t* targets, int ignore_index,
                                 float* lse, float* loss_mean, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
