// Allocation-free entry points of the bridge_b200 extension (C ABI).
//
// NOTE: these entry points have no counterpart in the reference implementation; they are an
// addition of this library.
//
// They serve callers that cannot allocate device memory at the point where the op runs: a C/C++
// host runtime that plans and owns every device allocation itself and hands kernels only its own
// buffers, or a training / serving loop that forbids allocation after start-up (a cudaMalloc can
// synchronize the device and stall the other streams).  The caller passes inputs and outputs; the
// FP32 scratch the kernel needs lives in a static device array of the library.
//
// Limits and behaviour (bb_rmsnorm_bwd_noalloc):
//   * 8 <= H <= BB_NOALLOC_MAX_HIDDEN and H % 8 == 0, rows >= 0; anything else returns
//     cudaErrorInvalidValue without launching, with a message in bb_noalloc_last_error().
//   * Scratch: BB_NOALLOC_SCRATCH_BYTES of static device memory, held by every GPU that loads the
//     library until the process exits.
//   * The first call on a device (that device current) resolves the scratch address once; make it
//     before any stream capture.  Host threads may call concurrently (the set-up runs once per device;
//     the error message is per thread).
//   * Calls share the scratch and it keeps the previous call's contents; each call overwrites what it
//     reads, so nothing has to be cleared.  Calls that overlap on the GPU (unordered streams) race on
//     the scratch: order them.
//   * No cudaMalloc, cudaFree or allocating library routine is called.
#ifndef BRIDGE_B200_NOALLOC_H_
#define BRIDGE_B200_NOALLOC_H_

#include <cuda_runtime.h>

#define BB_NOALLOC_SCRATCH_BYTES (4l << 20)
#define BB_NOALLOC_MAX_HIDDEN 32768

#ifdef __cplusplus
extern "C" {
#endif

// Message of the calling thread's last failed call (empty after a success).
const char* bb_noalloc_last_error(void);

// RMSNorm backward of y = x * rstd[row] * w: dx[rows, H] (bf16) and dw[H] (FP32, overwritten) from
// dy, x, w (bf16, row-major, contiguous) and rstd[rows] (FP32), enqueued on `stream`.
// Returns 0 (cudaSuccess) or a cudaError_t value.
int bb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                           long rows, int H, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif  // BRIDGE_B200_NOALLOC_H_
