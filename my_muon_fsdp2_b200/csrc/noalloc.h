// Allocation-free RMSNorm backward entry point (C ABI).
//
// This entry point has no counterpart in the reference project; it exists for callers of this
// library that cannot allocate device memory at the time they need the kernel — for example a
// C/C++ runtime that owns all device memory through its own pre-planned arena and forbids any
// cudaMalloc/cudaFree during a step (those calls may also synchronize the device), or code that
// is not linked against PyTorch's caching allocator at all.  Such callers pass only the inputs
// and outputs; the per-block partial sums that the regular path keeps in a freshly allocated
// buffer live instead in one fixed static device array (see noalloc.cu for its size), which
// every GPU that loads this library holds until the process exits.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest row width (number of columns) the scratch array is sized for.
#define MMF_NOALLOC_MAX_COLS 8192
// Maximum number of per-block partial rows kept in scratch (blocks launched <= this).
#define MMF_NOALLOC_MAX_PARTS 64

// dx = d(rmsnorm)/dx * dy and dw = sum over rows of dy * x * rstd, for bf16 dy, x, w, dx, dw
// and fp32 rstd (one value per row, as written by the forward pass).  x and dy are [rows, cols]
// row-major; w and dw have cols elements.  Returns 0 on success, or a non-zero code with a
// message from mmf_noalloc_last_error():
//   1: cols outside [1, MMF_NOALLOC_MAX_COLS] or rows < 1
//   2: scratch set-up failed (cudaGetSymbolAddress) on the current device
//   3: kernel launch failed (the message carries CUDA's error string)
//   4: `stream` belongs to another device than the current one (the scratch address is looked
//      up for the current device, so make the stream's device current before the call)
// The first call on each device looks up the scratch address with that device current; make
// that first call before any stream capture.  All calls share one scratch array per device
// and it keeps the last call's contents: calls that overlap on the GPU (different streams
// without ordering between them) race on it and must be serialised by the caller.
int mmf_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, void* dw,
                            int rows, int cols, cudaStream_t stream);

// Message for the last non-zero return code of this thread ("" if none).
const char* mmf_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
