// Symmetric peer memory over CUDA IPC, a cross-GPU barrier kernel, and the fused data-parallel
// optimizer path over NVLink / NVSwitch:
//
//   dp_reduce_scatter   each rank pulls ITS shard of every peer's FP32 gradient arena with P2P loads,
//                       sums in FP32 in fixed rank order, scales by 1/N and writes the result in place
//                       into its own arena (the shard nobody else reads), plus per-block sum-of-squares
//                       partials for the global gradient norm;
//   symm_barrier        (with payload) every rank pushes its norm partial into every peer's signal pad;
//   dp_adamw_allgather  AdamW on the local shard (clip from the N partials) and the new parameters
//                       stored straight into EVERY peer's parameter arena with 16-byte P2P stores.
//
// The bytes that cross NVLink per rank are (N-1)/N of the FP32 gradients in and (N-1)/N of the
// parameters out: a reduce-scatter + all-gather with the cast, scale, clip and optimizer fused in.
// Every wait is a bounded spin on %globaltimer; on timeout the kernel records the failing peer in
// an error word (read by the host) and returns.
//
// Parity: replaces the reference's Megatron finalize_model_grads(force_all_reduce=True) gradient
// all-reduce (verl/models/mcore/tpr/megatron_adapter.py:189-192, 457-461) and the replicated
// optimizer update after it.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstring>
#include <type_traits>

#include "common.cuh"

namespace {

constexpr int kMaxPeers = 8;
constexpr int kPadFlags = 0;      // uint64 flags[kMaxPeers]: flag j written by peer j
constexpr int kPadPayload = 64;   // double payload[kMaxPeers]: value j written by peer j
constexpr int kPadBytes = 256;

struct PeerPtrs {
  void* p[kMaxPeers];
};

__device__ unsigned int g_symm_error = 0;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One CTA of 32 threads; thread j signals peer j, then waits for peer j's signal.
__global__ void symm_barrier_kernel(PeerPtrs pads, int rank, int n, uint64_t epoch, const float* payload_src,
                                    int n_src, uint64_t timeout_ns) {
  __shared__ double val;
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < n_src; ++i) s += (double)payload_src[i];  // fixed order: deterministic
    val = s;
  }
  __syncthreads();
  const int j = threadIdx.x;
  if (j >= n) return;
  char* pad = static_cast<char*>(pads.p[j]);
  if (payload_src) *reinterpret_cast<volatile double*>(pad + kPadPayload + 8 * rank) = val;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  st_release_sys(reinterpret_cast<uint64_t*>(pad + kPadFlags) + rank, epoch);
  const uint64_t* mine = reinterpret_cast<const uint64_t*>(static_cast<char*>(pads.p[rank]) + kPadFlags) + j;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(mine) < epoch) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      atomicCAS(&g_symm_error, 0u, 0x100u + (unsigned)j);
      return;
    }
    __nanosleep(64);
  }
}

// Per-bucket readiness flags for the reduce-scatter overlapped with backward: flags live in a
// symmetric buffer laid out [peer][bucket] (uint64 epochs).  `signal` (1 warp, after the bucket's
// gradients on the compute stream) stores `epoch` into slot [rank][bucket] of every peer's buffer with
// release semantics; `wait` (1 warp, on the reduce-scatter stream) spins with acquire loads until
// every peer's slot of `bucket` reached `epoch`, bounded by `timeout_ns` (error word 0x200 + peer).
__global__ void dp_bucket_signal_kernel(PeerPtrs flags, int rank, int n, int max_buckets, int bucket,
                                        uint64_t epoch) {
  const int j = threadIdx.x;
  if (j >= n) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  st_release_sys(static_cast<uint64_t*>(flags.p[j]) + (size_t)rank * max_buckets + bucket, epoch);
}

__global__ void dp_bucket_wait_kernel(const uint64_t* __restrict__ mine, int n, int max_buckets, int bucket,
                                      uint64_t epoch, uint64_t timeout_ns) {
  const int j = threadIdx.x;
  if (j >= n) return;
  const uint64_t* slot = mine + (size_t)j * max_buckets + bucket;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(slot) < epoch) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      atomicCAS(&g_symm_error, 0u, 0x200u + (unsigned)j);
      return;
    }
    __nanosleep(256);
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ float block_sum_512(float v, float* red) {
  v = bb::warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) t = bb::warp_sum(t);
  return t;  // valid in thread 0
}

// out (own arena + shard offset) = scale * sum_r grads[r][shard]; partials[block] = sum out^2
__global__ void __launch_bounds__(512) dp_rs_kernel(PeerPtrs grads, int n, size_t off4, size_t cnt4, float scale,
                                                    float4* __restrict__ out, float* __restrict__ partials) {
  __shared__ float red[32];
  float sq = 0.f;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < cnt4; i += stride) {
    float4 v[kMaxPeers];
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < n) v[r] = reinterpret_cast<const float4*>(grads.p[r])[off4 + i];
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < n) {
        a.x += v[r].x;
        a.y += v[r].y;
        a.z += v[r].z;
        a.w += v[r].w;
      }
    a.x *= scale;
    a.y *= scale;
    a.z *= scale;
    a.w *= scale;
    sq += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    out[i] = a;
  }
  const float t = block_sum_512(sq, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

__device__ __forceinline__ void adamw8(float* w, float* m, float* v, const float* g, float clip, float lr, float b1,
                                       float b2, float eps, float wd, float bc1, float bc2) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float gg = g[e] * clip;
    m[e] = b1 * m[e] + (1.f - b1) * gg;
    v[e] = b2 * v[e] + (1.f - b2) * gg * gg;
    const float den = sqrtf(v[e] / bc2) + eps;
    w[e] = w[e] * (1.f - lr * wd) - lr * (m[e] / bc1) / den;
  }
}

// AdamW on this rank's shard; the new parameters go to every peer's arena (P2P stores, 16 B / 32 B).
template <typename TP>
__global__ void __launch_bounds__(256) dp_adamw_ag_kernel(float4* __restrict__ master, float4* __restrict__ m,
                                                          float4* __restrict__ v, const float4* __restrict__ grad,
                                                          PeerPtrs data, int n, size_t off8, size_t cnt8,
                                                          const double* __restrict__ norm_slots, float max_norm,
                                                          float lr, float b1, float b2, float eps, float wd,
                                                          float bc1, float bc2, float* __restrict__ norm_out) {
  double s = 0.0;
  for (int r = 0; r < n; ++r) s += norm_slots[r];
  const float norm = (float)sqrt(s);
  const float clip = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *norm_out = norm;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < cnt8; i += stride) {
    float w[8], mm[8], vv[8], g[8];
    *reinterpret_cast<float4*>(w) = master[2 * i];
    *reinterpret_cast<float4*>(w + 4) = master[2 * i + 1];
    *reinterpret_cast<float4*>(mm) = m[2 * i];
    *reinterpret_cast<float4*>(mm + 4) = m[2 * i + 1];
    *reinterpret_cast<float4*>(vv) = v[2 * i];
    *reinterpret_cast<float4*>(vv + 4) = v[2 * i + 1];
    *reinterpret_cast<float4*>(g) = grad[2 * i];
    *reinterpret_cast<float4*>(g + 4) = grad[2 * i + 1];
    adamw8(w, mm, vv, g, clip, lr, b1, b2, eps, wd, bc1, bc2);
    master[2 * i] = *reinterpret_cast<float4*>(w);
    master[2 * i + 1] = *reinterpret_cast<float4*>(w + 4);
    m[2 * i] = *reinterpret_cast<float4*>(mm);
    m[2 * i + 1] = *reinterpret_cast<float4*>(mm + 4);
    v[2 * i] = *reinterpret_cast<float4*>(vv);
    v[2 * i + 1] = *reinterpret_cast<float4*>(vv + 4);
    if constexpr (std::is_same<TP, float>::value) {
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r < n) {
          float4* dst = reinterpret_cast<float4*>(data.p[r]) + 2 * (off8 + i);
          dst[0] = *reinterpret_cast<float4*>(w);
          dst[1] = *reinterpret_cast<float4*>(w + 4);
        }
    } else {
      const bb::bf16x8 pk = bb::pack8(w);
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r < n) reinterpret_cast<bb::bf16x8*>(data.p[r])[off8 + i] = pk;
    }
  }
}

PeerPtrs make_ptrs(const std::vector<int64_t>& v) {
  TORCH_CHECK(!v.empty() && v.size() <= (size_t)kMaxPeers, "symmetric memory: 1..8 peers");
  PeerPtrs p{};
  for (size_t i = 0; i < v.size(); ++i) {
    TORCH_CHECK(v[i] != 0 && v[i] % 16 == 0, "symmetric memory: peer pointer must be 16-byte aligned");
    p.p[i] = reinterpret_cast<void*>(v[i]);
  }
  return p;
}

int num_blocks(size_t work, int threads, int per_sm) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t need = (work + threads - 1) / threads;
  return (int)std::max<size_t>(1, std::min<size_t>(need, (size_t)sms * per_sm));
}

}  // namespace

// ---------------------------------------------------------------------------------------- host API
std::vector<torch::Tensor> symm_alloc(int64_t nbytes) {
  TORCH_CHECK(nbytes > 0, "symm_alloc: size must be positive");
  const int dev = c10::cuda::current_device();
  void* ptr = nullptr;
  BB_CHECK_CUDA(cudaMalloc(&ptr, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  BB_CHECK_CUDA(cudaIpcGetMemHandle(&h, ptr));
  auto local = torch::from_blob(
      ptr, {nbytes}, [](void* p) { cudaFree(p); },
      torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, dev));
  auto handle = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(handle.data_ptr(), &h, sizeof(h));
  return {local, handle};
}

int64_t symm_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && !handle.is_cuda(), "symm_open: bad handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* ptr = nullptr;
  BB_CHECK_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void symm_close(int64_t ptr) { BB_CHECK_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

int64_t symm_pad_bytes() { return kPadBytes; }

void symm_barrier(std::vector<int64_t> pads, int64_t rank, int64_t epoch, c10::optional<torch::Tensor> payload,
                  double timeout_s) {
  const int n = (int)pads.size();
  TORCH_CHECK(rank >= 0 && rank < n, "symm_barrier: rank out of range");
  const float* src = nullptr;
  int n_src = 0;
  if (payload.has_value()) {
    TORCH_CHECK(payload->is_cuda() && payload->scalar_type() == at::kFloat && payload->is_contiguous(),
                "symm_barrier: payload must be contiguous fp32 on the device");
    src = payload->data_ptr<float>();
    n_src = (int)payload->numel();
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  symm_barrier_kernel<<<1, 32, 0, stream>>>(make_ptrs(pads), (int)rank, n, (uint64_t)epoch, src, n_src,
                                            (uint64_t)(timeout_s * 1e9));
  BB_POST_LAUNCH();
}

void dp_reduce_scatter(std::vector<int64_t> grads, int64_t rank, int64_t offset, int64_t count, double scale,
                       torch::Tensor partials) {
  const int n = (int)grads.size();
  TORCH_CHECK(offset % 4 == 0 && count % 4 == 0, "dp_reduce_scatter: offset/count must be multiples of 4");
  TORCH_CHECK(partials.is_cuda() && partials.scalar_type() == at::kFloat, "dp_reduce_scatter: fp32 partials");
  const int blocks = std::min<int>(num_blocks(count / 4, 512, 4), (int)partials.numel());
  partials.zero_();
  auto stream = at::cuda::getCurrentCUDAStream();
  float4* out = reinterpret_cast<float4*>(grads[rank]) + offset / 4;
  dp_rs_kernel<<<blocks, 512, 0, stream>>>(make_ptrs(grads), n, (size_t)(offset / 4), (size_t)(count / 4),
                                           (float)scale, out, partials.data_ptr<float>());
  BB_POST_LAUNCH();
}

void dp_adamw_allgather(torch::Tensor master, torch::Tensor m, torch::Tensor v, torch::Tensor grad_shard,
                        std::vector<int64_t> data, int64_t offset, bool bf16_params, int64_t pad_ptr, double max_norm,
                        double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                        torch::Tensor norm_out) {
  const int64_t cnt = master.numel();
  TORCH_CHECK(cnt % 8 == 0 && offset % 8 == 0, "dp_adamw_allgather: shard must be a multiple of 8 elements");
  for (auto* t : {&master, &m, &v, &grad_shard})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == cnt,
                "dp_adamw_allgather: fp32 contiguous shard tensors of equal size");
  const int n = (int)data.size();
  const int blocks = num_blocks(cnt / 8, 256, 8);
  auto stream = at::cuda::getCurrentCUDAStream();
  const double* slots = reinterpret_cast<const double*>(reinterpret_cast<char*>(pad_ptr) + kPadPayload);
#define BB_AG(T)                                                                                                 \
  dp_adamw_ag_kernel<T><<<blocks, 256, 0, stream>>>(                                                             \
      reinterpret_cast<float4*>(master.data_ptr<float>()), reinterpret_cast<float4*>(m.data_ptr<float>()),         \
      reinterpret_cast<float4*>(v.data_ptr<float>()), reinterpret_cast<const float4*>(grad_shard.data_ptr<float>()), \
      make_ptrs(data), n, (size_t)(offset / 8), (size_t)(cnt / 8), slots, (float)max_norm, (float)lr, (float)b1,    \
      (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2, norm_out.data_ptr<float>())
  if (bf16_params) BB_AG(__nv_bfloat16);
  else BB_AG(float);
#undef BB_AG
  BB_POST_LAUNCH();
}

void dp_bucket_signal(std::vector<int64_t> flags, int64_t rank, int64_t max_buckets, int64_t bucket, int64_t epoch) {
  TORCH_CHECK(bucket >= 0 && bucket < max_buckets && rank >= 0 && rank < (int64_t)flags.size(),
              "dp_bucket_signal: bucket / rank out of range");
  dp_bucket_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      make_ptrs(flags), (int)rank, (int)flags.size(), (int)max_buckets, (int)bucket, (uint64_t)epoch);
  BB_POST_LAUNCH();
}

void dp_bucket_wait(int64_t mine, int64_t n, int64_t max_buckets, int64_t bucket, int64_t epoch, double timeout_s) {
  TORCH_CHECK(mine != 0 && mine % 16 == 0 && n >= 1 && n <= kMaxPeers && bucket >= 0 && bucket < max_buckets,
              "dp_bucket_wait: bad flag buffer, peer count or bucket");
  dp_bucket_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint64_t*>(mine), (int)n, (int)max_buckets, (int)bucket, (uint64_t)epoch,
      (uint64_t)(timeout_s * 1e9));
  BB_POST_LAUNCH();
}

// dst[0:nbytes) = *src_ptr (a peer's symmetric buffer, or any device address) by the copy engine on the
// current stream: the NVLink transfer takes no SMs away from a concurrently running GEMM.
void p2p_copy(torch::Tensor dst, int64_t src_ptr, int64_t nbytes) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous() && nbytes >= 0 &&
                  nbytes <= (int64_t)(dst.numel() * dst.element_size()) && src_ptr != 0,
              "p2p_copy: contiguous CUDA dst of at least nbytes and a non-null source");
  if (nbytes == 0) return;
  BB_CHECK_CUDA(cudaMemcpyAsync(dst.data_ptr(), reinterpret_cast<const void*>(src_ptr), (size_t)nbytes,
                                cudaMemcpyDeviceToDevice, at::cuda::getCurrentCUDAStream()));
}

int64_t symm_error_code() {
  unsigned int v = 0;
  BB_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_symm_error, sizeof(v)));
  return v;
}

void symm_clear_error() {
  const unsigned int z = 0;
  BB_CHECK_CUDA(cudaMemcpyToSymbol(g_symm_error, &z, sizeof(z)));
}

// ------------------------------------------------------------------------------------------------
// Row-indexed P2P movement over symmetric buffers (context-parallel KV exchange, MoE dispatch):
//   p2p_gather_rows  out[i, :] = peer[src_rank[i]][src_row[i], :]              (bf16 rows)
//   p2p_reduce_rows  out[i, :] = sum_r peer[r][src_row[i], :]  (+ add[i, :])    (bf16 or fp32 rows,
//                    fixed rank order, FP32 accumulation, bf16 or fp32 out)
// One warp per row, 16-byte vectors, several loads in flight per lane.
namespace {

__global__ void p2p_gather_rows_kernel(PeerPtrs peers, const int* __restrict__ src_rank,
                                       const int* __restrict__ src_row, uint4* __restrict__ out, int rows,
                                       int vecs /* 16-byte vectors per row */) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  for (int i = gw; i < rows; i += nw) {
    const int r = src_rank[i];
    const uint4* src = reinterpret_cast<const uint4*>(peers.p[r]) + (size_t)src_row[i] * vecs;
    uint4* dst = out + (size_t)i * vecs;
    for (int v0 = 0; v0 < vecs; v0 += 32 * 4) {
      uint4 buf[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v < vecs) buf[u] = __ldg(src + v);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * 32 + lane;
        if (v < vecs) dst[v] = buf[u];
      }
    }
  }
}

template <bool SRC_F32, bool OUT_F32>
__global__ void p2p_reduce_rows_kernel(PeerPtrs peers, int n, const int* __restrict__ src_row,
                                       const bb::bf16x8* __restrict__ add, void* __restrict__ out_raw, int rows,
                                       int vecs /* 8-element vectors per row */) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  for (int i = gw; i < rows; i += nw) {
    const size_t srow = (size_t)src_row[i] * vecs;
    for (int v = lane; v < vecs; v += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (add) bb::unpack8(add[(size_t)i * vecs + v], acc);
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r) {
        if (r >= n) break;
        float f[8];
        if (SRC_F32) {
          const float4* s = reinterpret_cast<const float4*>(peers.p[r]) + 2 * (srow + v);
          const float4 a = __ldg(s), b = __ldg(s + 1);
          f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        } else {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(peers.p[r]) + srow + v);
          bb::unpack8(*reinterpret_cast<const bb::bf16x8*>(&raw), f);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += f[e];
      }
      if (OUT_F32) {
        float4* o = reinterpret_cast<float4*>(out_raw) + 2 * ((size_t)i * vecs + v);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      } else {
        reinterpret_cast<bb::bf16x8*>(out_raw)[(size_t)i * vecs + v] = bb::pack8(acc);
      }
    }
  }
}

}  // namespace

void p2p_gather_rows(torch::Tensor out, std::vector<int64_t> peers, torch::Tensor src_rank, torch::Tensor src_row) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.dim() == 2, "p2p_gather_rows: out [rows, width]");
  const int64_t row_bytes = out.size(1) * out.element_size();
  TORCH_CHECK(row_bytes % 16 == 0, "p2p_gather_rows: row bytes must be a multiple of 16");
  const int rows = (int)out.size(0);
  TORCH_CHECK(src_rank.numel() == rows && src_row.numel() == rows && src_rank.scalar_type() == at::kInt &&
                  src_row.scalar_type() == at::kInt && src_rank.is_cuda(),
              "p2p_gather_rows: int32 index tensors of out.size(0) on the device");
  if (rows == 0) return;
  const int blocks = num_blocks((size_t)rows * 32, 256, 8);
  p2p_gather_rows_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      make_ptrs(peers), src_rank.data_ptr<int>(), src_row.data_ptr<int>(), reinterpret_cast<uint4*>(out.data_ptr()),
      rows, (int)(row_bytes / 16));
  BB_POST_LAUNCH();
}

void p2p_reduce_rows(torch::Tensor out, std::vector<int64_t> peers, torch::Tensor src_row, bool src_f32,
                     c10::optional<torch::Tensor> add) {
  const bool out_f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.dim() == 2 &&
                  (out.scalar_type() == at::kBFloat16 || out_f32),
              "p2p_reduce_rows: bf16 or fp32 out [rows, width]");
  TORCH_CHECK(!out_f32 || src_f32, "p2p_reduce_rows: an fp32 out needs fp32 source rows");
  TORCH_CHECK(out.size(1) % 8 == 0, "p2p_reduce_rows: width must be a multiple of 8");
  const int rows = (int)out.size(0);
  TORCH_CHECK(src_row.numel() == rows && src_row.scalar_type() == at::kInt && src_row.is_cuda(),
              "p2p_reduce_rows: int32 row index on the device");
  const bb::bf16x8* addp = nullptr;
  if (add.has_value()) {
    TORCH_CHECK(!out_f32 && add->is_contiguous() && add->scalar_type() == at::kBFloat16 &&
                    add->numel() == out.numel(),
                "p2p_reduce_rows: add must match a bf16 out");
    addp = reinterpret_cast<const bb::bf16x8*>(add->data_ptr());
  }
  if (rows == 0) return;
  const int blocks = num_blocks((size_t)rows * 32, 256, 8);
  auto stream = at::cuda::getCurrentCUDAStream();
  void* o = out.data_ptr();
  const int vecs = (int)(out.size(1) / 8);
  const int np = (int)peers.size();
  if (out_f32)
    p2p_reduce_rows_kernel<true, true><<<blocks, 256, 0, stream>>>(make_ptrs(peers), np, src_row.data_ptr<int>(),
                                                                   addp, o, rows, vecs);
  else if (src_f32)
    p2p_reduce_rows_kernel<true, false><<<blocks, 256, 0, stream>>>(make_ptrs(peers), np, src_row.data_ptr<int>(),
                                                                    addp, o, rows, vecs);
  else
    p2p_reduce_rows_kernel<false, false><<<blocks, 256, 0, stream>>>(make_ptrs(peers), np, src_row.data_ptr<int>(),
                                                                     addp, o, rows, vecs);
  BB_POST_LAUNCH();
}
