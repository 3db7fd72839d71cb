// Allocation-free C entry point of the RMSNorm backward kernel.
//
// This entry point has no counterpart in the reference implementation.  It exists for
// callers that cannot allocate device memory at call time: for example a host
// application whose device memory is owned by its own pool allocator (a raw cudaMalloc
// or cudaFree would bypass that pool's accounting, and cudaFree can synchronize the whole
// device), or code that is handed raw pointers and is not allowed to allocate.  Such a
// caller passes its inputs and outputs; the kernel's scratch space (one partial row of
// the weight gradient per thread block) lives in a fixed, file-scope device array of
// NSW_NOALLOC_RMSNORM_PARTS x NSW_NOALLOC_RMSNORM_MAX_N floats (1 MiB), which every GPU
// that loads the library holds until the process exits.
//
// Behaviour:
//   * The first call on a device looks up the device address of that array
//     (cudaGetSymbolAddress, with that device current); make that first call before any
//     stream capture.  Later calls on the same device reuse the address.
//   * Nothing is allocated or freed: no cudaMalloc, cudaFree or allocating library call.
//   * Every call shares the one array, which keeps the previous call's contents.  Each call
//     writes every partial row it later reads, so nothing needs clearing, but two calls
//     that overlap on the GPU (for example on different streams) race on the array and
//     give wrong results: serialise them.
//   * n (the normalised size) must be a multiple of 8 and at most
//     NSW_NOALLOC_RMSNORM_MAX_N; larger sizes are rejected with NSW_NOALLOC_ERR_TOO_LARGE
//     before anything is launched.
//   * dy, x and dx are accessed 16 bytes at a time: their addresses must be multiples of
//     16 bytes (a row offset into a larger buffer must keep that), otherwise the call
//     returns NSW_NOALLOC_ERR_BAD_ARG.
//   * rows == 0 writes zeros to dw (an asynchronous memset on the stream) and launches
//     no kernel.
//   * If a CUDA error from an earlier call on this thread is still pending, the call
//     returns NSW_NOALLOC_ERR_PENDING and launches nothing (the pending error is left for
//     the caller to read), so that NSW_NOALLOC_ERR_LAUNCH always means this call's launch.
#pragma once

#include <stdint.h>

#define NSW_NOALLOC_RMSNORM_MAX_N 2048
#define NSW_NOALLOC_RMSNORM_PARTS 128

#define NSW_NOALLOC_OK 0
#define NSW_NOALLOC_ERR_TOO_LARGE 1001
#define NSW_NOALLOC_ERR_BAD_ARG 1002
#define NSW_NOALLOC_ERR_SYMBOL 1003
#define NSW_NOALLOC_ERR_LAUNCH 1004
#define NSW_NOALLOC_ERR_PENDING 1005

#ifdef __cplusplus
extern "C" {
#endif

// Gradients of y = x * rstd * w (rows x n, row-major) given dy:
//   dx[r, :] = rstd[r] * (dy*w - xhat * mean(dy * w * xhat)),  xhat = x * rstd[r]
//   dw[:]    = sum_r dy[r, :] * xhat[r, :]                     (fp32, written, not added)
// dtype: 0 = bf16, 1 = fp16 for dy, x and dx; w, rstd and dw are fp32.  stream is a
// cudaStream_t (0 for the legacy default stream).  Returns NSW_NOALLOC_OK or an error code.
int nsw_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                            float* dw, int64_t rows, int n, int dtype, void* stream);

// Human-readable text of an error code returned above.
const char* nsw_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
