// Allocation-free column sums: one extern "C" entry point.
//
// This entry point has no counterpart in the reference framework.
//
// Why it exists: some callers of this library cannot allocate device memory
// at the moment they need the reduction -- a host application that runs
// inside a strict memory budget and forbids allocations after start-up, a
// plugin called by a runtime that owns all device memory, or code running on
// a thread where a cudaMalloc (which can synchronise the device) would stall
// latency-critical work.  The regular entry point (dlvk::colsum) takes a
// caller-provided scratch buffer that its PyTorch binding allocates; this one
// needs nothing from the caller except the input and the output.
//
// Scratch: a file-scope __device__ array of DLVK_NOALLOC_SCRATCH_FLOATS floats
// (4 MiB).  Every GPU that loads this library holds that array until the
// process exits.  It holds up to 64 row-chunk partials per column, so at most
// DLVK_NOALLOC_MAX_COLS columns are accepted; larger requests are rejected
// with DLVK_NOALLOC_TOO_LARGE before anything is launched.
//
// The first call on each device looks up the array's device address
// (cudaGetSymbolAddress, with that device current) and caches it; make that
// first call before any CUDA-graph stream capture on the device.  All calls
// share the one array and every call rewrites the parts of it that it reads,
// so it keeps the last call's partial sums and needs no clearing; calls that
// overlap on the GPU (different streams without ordering) race on it.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#define DLVK_NOALLOC_SCRATCH_FLOATS (1 << 20)
#define DLVK_NOALLOC_MAX_COLS (DLVK_NOALLOC_SCRATCH_FLOATS / 64)

#define DLVK_NOALLOC_OK 0
#define DLVK_NOALLOC_BAD_ARG 1
#define DLVK_NOALLOC_TOO_LARGE 2
#define DLVK_NOALLOC_CUDA_ERROR 3

#ifdef __cplusplus
extern "C" {
#endif

// out[c] = scale * sum_r x[r * cols + c] (+ out[c] if accumulate != 0).
// x: device pointer, dtype 0 = float32, 1 = bfloat16, row-major [rows, cols];
// out: device float32 [cols].  Enqueued on `stream`; returns a
// DLVK_NOALLOC_* code.  Allocates no memory.  DLVK_NOALLOC_CUDA_ERROR is
// also returned, before anything is launched, when an earlier CUDA error is
// already pending on the calling thread; in every error case `out` has not
// been written by this call.
int dlvk_colsum_noalloc(const void* x, int dtype, int64_t rows, int64_t cols, float scale, float* out,
                        int accumulate, cudaStream_t stream);

// Human-readable text for a DLVK_NOALLOC_* code.
const char* dlvk_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
