// RMSNorm backward that allocates nothing: C entry point for callers that cannot allocate.
//
// NOTE: this entry point has no counterpart in the reference implementation; it is an addition of
// this library.
//
// Who needs it.  Some callers cannot call cudaMalloc (or torch's caching allocator) at the point
// where they run this op: a C/C++ host runtime that owns every device allocation itself and hands
// kernels only pre-planned buffers, or a serving / training loop that forbids allocation after
// start-up because a cudaMalloc can synchronize the device and stall the other streams.  Such a
// caller passes its inputs and outputs; the FP32 reduction scratch this kernel needs lives in a
// fixed static device array instead of a per-call allocation.
//
// Contract.
//   * Scratch: `g_noalloc_rms_scratch`, kNoAllocScratchFloats FP32 values (4 MiB).  Every GPU that
//     loads this library holds it until the process exits.
//   * Limits: 8 <= H <= 32768 with H % 8 == 0.  The kernel uses nblocks x H scratch floats and picks
//     nblocks so that it fits; H above the limit is rejected (cudaErrorInvalidValue, nothing launched,
//     message available from bb_noalloc_last_error()).
//   * The first call on a device, with that device current, resolves the device address of the
//     scratch array (cudaGetSymbolAddress) and caches it per device.  Make that first call before any
//     stream capture.
//   * Every call shares the one array and it keeps the previous call's contents.  Each call fully
//     overwrites the part it reads, so nothing has to start at zero; but calls that overlap on the
//     GPU (different streams without ordering) race on the scratch and must be serialized by the
//     caller.
//   * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

namespace {

constexpr long kNoAllocScratchFloats = 1l << 20;  // 4 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_rms_scratch[kNoAllocScratchFloats];

float* g_scratch_ptr[kMaxDevices] = {nullptr};
char g_last_error[256] = "";

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row; per-block FP32 partial weight-gradient row written to scratch[block].
__global__ void rms_bwd_partial(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                __nv_bfloat16* __restrict__ dx, float* __restrict__ part, long rows, int H) {
  extern __shared__ float sdw[];
  for (int i = threadIdx.x; i < H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long row = (long)blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += (long)gridDim.x * warps) {
    const __nv_bfloat16* xr = x + row * H;
    const __nv_bfloat16* gr = dy + row * H;
    const float r = rstd[row];
    float dot = 0.f;
    for (int i = lane; i < H; i += 32) dot += __bfloat162float(gr[i]) * __bfloat162float(w[i]) * __bfloat162float(xr[i]) * r;
    dot = wsum(dot) / H;
    for (int i = lane; i < H; i += 32) {
      const float xv = __bfloat162float(xr[i]), gv = __bfloat162float(gr[i]), wv = __bfloat162float(w[i]);
      dx[row * H + i] = __float2bfloat16(r * (gv * wv - xv * r * dot));
      atomicAdd(&sdw[i], gv * xv * r);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) part[(long)blockIdx.x * H + i] = sdw[i];
}

__global__ void rms_bwd_colsum(const float* __restrict__ part, float* __restrict__ dw, int nblocks, int H) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int b = 0; b < nblocks; ++b) s += part[(long)b * H + c];
  dw[c] = s;
}

int fail(cudaError_t e, const char* msg) {
  snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return (int)e;
}

}  // namespace

extern "C" {

// Last error message of the no-allocation entry points (empty after a successful call).
const char* bb_noalloc_last_error() { return g_last_error; }

// dx[rows, H] (bf16) and dw[H] (FP32, overwritten) of y = x * rstd * w given dy, x, w, rstd.
// Returns 0 (cudaSuccess) or a cudaError_t value; see the contract at the top of this file.
int bb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                           long rows, int H, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (H < 8 || H > 32768 || (H % 8) != 0)
    return fail(cudaErrorInvalidValue, "bb_rmsnorm_bwd_noalloc: H must be a multiple of 8 in [8, 32768]");
  if (rows < 0) return fail(cudaErrorInvalidValue, "bb_rmsnorm_bwd_noalloc: rows must be >= 0");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "bb_rmsnorm_bwd_noalloc: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return fail(cudaErrorInvalidDevice, "bb_rmsnorm_bwd_noalloc: device index");
  if (g_scratch_ptr[dev] == nullptr) {
    // One-time set-up on this device (the device is current): host code may not use the symbol
    // itself as a device address, so resolve it.
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_rms_scratch);
    if (e != cudaSuccess || p == nullptr) return fail(e, "bb_rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed");
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  if (rows == 0) {
    e = cudaMemsetAsync(dw, 0, sizeof(float) * (size_t)H, stream);
    return e == cudaSuccess ? 0 : fail(e, "bb_rmsnorm_bwd_noalloc: memset failed");
  }
  const int threads = 256, warps = threads / 32;
  long want = (rows + warps - 1) / warps;
  long cap = kNoAllocScratchFloats / H;  // partial rows that fit in the scratch array
  int nblocks = (int)(want < cap ? want : cap);
  if (nblocks > 512) nblocks = 512;
  if (nblocks < 1) return fail(cudaErrorInvalidValue, "bb_rmsnorm_bwd_noalloc: H exceeds the scratch size");
  const size_t smem = sizeof(float) * (size_t)H;
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(rms_bwd_partial, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(e, "bb_rmsnorm_bwd_noalloc: shared-memory attribute");
  }
  rms_bwd_partial<<<nblocks, threads, smem, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
      rstd, static_cast<__nv_bfloat16*>(dx), g_scratch_ptr[dev], rows, H);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(e, "bb_rmsnorm_bwd_noalloc: partial kernel launch failed");
  rms_bwd_colsum<<<(H + 255) / 256, 256, 0, stream>>>(g_scratch_ptr[dev], dw, nblocks, H);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(e, "bb_rmsnorm_bwd_noalloc: column-sum kernel launch failed");
  return 0;
}

}  // extern "C"
