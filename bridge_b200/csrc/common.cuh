// Shared device helpers for the bridge_b200 sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define BB_CHECK_CUDA(expr)                                                                    \
  do {                                                                                         \
    cudaError_t _e = (expr);                                                                   \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__, \
                ":", __LINE__);                                                                \
  } while (0)

namespace bb {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 8 x bf16 <-> 16-byte vector
struct alignas(16) bf16x8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const bf16x8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ bf16x8 pack8(const float* f) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

// Block-wide sum over all threads (blockDim.x multiple of 32, <= 1024); result valid in every thread.
__device__ __forceinline__ float block_sum(float v, float* scratch /* >= 32 floats */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? scratch[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

}  // namespace bb

#include <atomic>
namespace bb {
// Number of kernels this extension has launched (read by benchmarks to report gpu_launches).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> c{0};
  return c;
}
}  // namespace bb
namespace bb {
// Grid for a grid-stride kernel: at most the number of blocks that are resident at once on all SMs
// (a larger grid would run as a partial second wave), and no more than `want`.
template <typename Kernel>
inline int resident_grid(Kernel kernel, int threads, size_t smem, long want) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  const long cap = (long)sms * (per_sm > 0 ? per_sm : 1);
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}
}  // namespace bb
namespace bb {
// Sets a kernel's dynamic shared-memory limit once per device (the attribute is per-device state:
// a process that drives several GPUs must set it on each).
template <typename Kernel>
inline void set_smem_attr_once(Kernel kernel, int smem, unsigned long long& done_mask) {
  int dev = 0;
  BB_CHECK_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (done_mask & bit) return;
  BB_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  done_mask |= bit;
}
}  // namespace bb
#define BB_POST_LAUNCH()                  \
  do {                                    \
    BB_CHECK_CUDA(cudaGetLastError());    \
    bb::launch_counter().fetch_add(1);    \
  } while (0)
