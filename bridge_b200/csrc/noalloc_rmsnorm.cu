// RMSNorm backward that allocates nothing: the C entry point declared in noalloc.h (which states
// who needs it, its limits and its contract).
//
// NOTE: this entry point has no counterpart in the reference implementation; it is an addition of
// this library.
//
// The FP32 weight-gradient partials live in `g_noalloc_rms_scratch` (BB_NOALLOC_SCRATCH_BYTES).  The
// partial kernel uses nblocks x H of it and nblocks is capped so that it fits.  Host code must not use
// the array's name as a device address: the first call on each device resolves it with
// cudaGetSymbolAddress (once per device, std::call_once) and every call passes that pointer.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "noalloc.h"

namespace {

constexpr long kNoAllocScratchFloats = BB_NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_rms_scratch[kNoAllocScratchFloats];

std::once_flag g_scratch_once[kMaxDevices];
std::atomic<float*> g_scratch_ptr[kMaxDevices];
std::atomic<int> g_scratch_err[kMaxDevices];
thread_local char g_last_error[256] = "";

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

const char* bb_noalloc_last_error(void) { return g_last_error; }

int bb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                           long rows, int H, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (H < 8 || H > BB_NOALLOC_MAX_HIDDEN || (H % 8) != 0)
    return fail(cudaErrorInvalidValue, "bb_rmsnorm_bwd_noalloc: H must be a multiple of 8 in [8, 32768]");
  if (rows < 0) return fail(cudaErrorInvalidValue, "bb_rmsnorm_bwd_noalloc: rows must be >= 0");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "bb_rmsnorm_bwd_noalloc: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return fail(cudaErrorInvalidDevice, "bb_rmsnorm_bwd_noalloc: device index");
  // One-time set-up on this device (the device is current): host code may not use the symbol itself
  // as a device address, so resolve it.  call_once makes concurrent first calls from several host
  // threads safe.
  std::call_once(g_scratch_once[dev], [dev]() {
    void* p = nullptr;
    const cudaError_t se = cudaGetSymbolAddress(&p, g_noalloc_rms_scratch);
    g_scratch_err[dev].store(se == cudaSuccess && p == nullptr ? (int)cudaErrorInvalidSymbol : (int)se);
    g_scratch_ptr[dev].store(static_cast<float*>(p));
  });
  float* scratch = g_scratch_ptr[dev].load();
  if (scratch == nullptr) {
    const int se = g_scratch_err[dev].load();
    return fail(se ? (cudaError_t)se : cudaErrorInvalidSymbol, "bb_rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed");
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
      rstd, static_cast<__nv_bfloat16*>(dx), scratch, rows, H);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(e, "bb_rmsnorm_bwd_noalloc: partial kernel launch failed");
  rms_bwd_colsum<<<(H + 255) / 256, 256, 0, stream>>>(scratch, dw, nblocks, H);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(e, "bb_rmsnorm_bwd_noalloc: column-sum kernel launch failed");
  return 0;
}

}  // extern "C"
