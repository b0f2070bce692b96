// MoE routing and combine on the device (Qwen3-Next form: softmax over all experts, top-k,
// renormalised; the global softmax denominator cancels, so the kept weights are a softmax over the
// k selected logits).
//
//   moe_route     logits [T, E] (fp32) -> idx [T, k] (int32), w [T, k] (fp32), counts [E] (int32),
//                 offsets [E + 1] (int32, exclusive scan), pos [T * k] (int32: where routed row
//                 (t, j) sits in the expert-sorted order), order [T * k] (int32: the inverse, the flat
//                 (t * k + j) index of each sorted row).  One warp per token for the top-k (each lane
//                 holds E / 32 logits in registers; k rounds of a warp arg-max, ties to the lower
//                 expert id), a shared-memory histogram, a one-block scan, then one pass that places
//                 every routed row.  Rows inside an expert come out in token order (a stable counting
//                 sort: block b's rows of expert e follow those of blocks < b, and inside a block the
//                 warp ballots keep token order).
//   moe_combine   y [T, H] = sum_j w[t, j] * ys[pos[t * k + j]]  (FP32 accumulate, no atomics)
//   moe_combine_bwd  dys[pos[t * k + j]] = w[t, j] * dy[t];  dw[t, j] = <dy[t], ys[pos[t * k + j]]>
//   moe_route_bwd    dlogits[t, e] = w_j (dw_j - sum_i w_i dw_i) for the k selected e, 0 elsewhere
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace {

constexpr int kMaxPerLane = 32;   // E <= 1024
constexpr int kMaxTopK = 32;

template <int PER_LANE>
__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ logits, int T, int E, int k,
                                                   int* __restrict__ idx, float* __restrict__ w) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    float v[PER_LANE];
    const float* row = logits + (size_t)t * E;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = i * 32 + lane;
      v[i] = e < E ? row[e] : -INFINITY;
    }
    float sel_v[kMaxTopK];
    int sel_e[kMaxTopK];
    for (int j = 0; j < k; ++j) {
      float best = -INFINITY;
      int be = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int e = i * 32 + lane;
        if (v[i] > best || (v[i] == best && e < be)) {
          best = v[i];
          be = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (ob > best || (ob == best && oe < be)) {
          best = ob;
          be = oe;
        }
      }
      sel_v[j] = best;
      sel_e[j] = be;
      if ((be & 31) == lane) {
#pragma unroll
        for (int i = 0; i < PER_LANE; ++i)
          if (i == (be >> 5)) v[i] = -INFINITY;
      }
    }
    // softmax over the k kept logits (sel_v[0] is their maximum)
    float s = 0.f;
    for (int j = 0; j < k; ++j) s += __expf(sel_v[j] - sel_v[0]);
    const float inv = 1.f / s;
    for (int j = lane; j < k; j += 32) {
      // every lane holds the same sel arrays; lane j writes entry j
      float vj = sel_v[0];
      int ej = sel_e[0];
      for (int q = 0; q < k; ++q)
        if (q == j) {
          vj = sel_v[q];
          ej = sel_e[q];
        }
      idx[(size_t)t * k + j] = ej;
      w[(size_t)t * k + j] = __expf(vj - sel_v[0]) * inv;
    }
  }
}

// Per-block expert histograms (block b counts rows [b * chunk, (b + 1) * chunk) of the flat idx).
__global__ void __launch_bounds__(256) block_hist_kernel(const int* __restrict__ idx, long n, int E, long chunk,
                                                         int* __restrict__ block_counts /* [nb, E] */) {
  extern __shared__ int h[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const long lo = (long)blockIdx.x * chunk, hi = min(n, lo + chunk);
  for (long i = lo + threadIdx.x; i < hi; i += blockDim.x) atomicAdd(&h[idx[i]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_counts[(size_t)blockIdx.x * E + e] = h[e];
}

// One block: counts[e] = sum_b block_counts[b, e]; offsets = exclusive scan of counts; block_base[b, e]
// = offsets[e] + sum_{b' < b} block_counts[b', e].
__global__ void __launch_bounds__(1024) scan_kernel(int* __restrict__ block_counts, int nb, int E,
                                                    int* __restrict__ counts, int* __restrict__ offsets) {
  __shared__ int tot[1024];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < nb; ++b) {
      const int c = block_counts[(size_t)b * E + e];
      block_counts[(size_t)b * E + e] = run;     // becomes the per-block base inside expert e
      run += c;
    }
    counts[e] = run;
    tot[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = acc;
      acc += tot[e];
    }
    offsets[E] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    for (int b = 0; b < nb; ++b) block_counts[(size_t)b * E + e] += offsets[e];
}

// Place every routed row.  A block walks its chunk in rounds of blockDim rows; inside a warp the
// rows of one expert are ranked with __match_any_sync, and the warps of a round take their slots in
// warp order (the last row of each same-expert group advances that expert's cursor), so slots follow
// row order: a stable counting sort.
__global__ void __launch_bounds__(256) place_kernel(const int* __restrict__ idx, long n, int E, long chunk,
                                                    const int* __restrict__ block_base, int* __restrict__ pos,
                                                    int* __restrict__ order) {
  extern __shared__ int cursor[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = block_base[(size_t)blockIdx.x * E + e];
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const unsigned lt = (1u << lane) - 1u;
  const long lo = (long)blockIdx.x * chunk, hi = min(n, lo + chunk);
  for (long base = lo; base < hi; base += blockDim.x) {
    const long i = base + threadIdx.x;
    const bool valid = i < hi;
    const int e = valid ? idx[i] : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(grp & lt), cnt = __popc(grp);
    for (int ww = 0; ww < nw; ++ww) {
      int slot = 0;
      if (wid == ww && valid) {
        slot = cursor[e] + rank;
        pos[i] = slot;
        order[slot] = (int)i;
      }
      __syncthreads();                       // every member read the cursor
      if (wid == ww && valid && rank == cnt - 1) cursor[e] += cnt;
      __syncthreads();
      (void)slot;
    }
  }
}

__global__ void __launch_bounds__(256) combine_fwd_kernel(const __nv_bfloat16* __restrict__ ys,
                                                          const int* __restrict__ pos, const float* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y, int T, int H, int k) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  const int vecs = H / 8;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    for (int v = lane; v < vecs; v += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < k; ++j) {
        const int p = pos[(size_t)t * k + j];
        const float g = w[(size_t)t * k + j];
        float f[8];
        bb::unpack8(reinterpret_cast<const bb::bf16x8*>(ys + (size_t)p * H)[v], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += g * f[e];
      }
      reinterpret_cast<bb::bf16x8*>(y + (size_t)t * H)[v] = bb::pack8(acc);
    }
  }
}

// One warp per routed row (t, j).
__global__ void __launch_bounds__(256) combine_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                          const __nv_bfloat16* __restrict__ ys,
                                                          const int* __restrict__ pos, const float* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ dys, float* __restrict__ dw,
                                                          long n, int H, int k) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  const int vecs = H / 8;
  for (long r = (long)blockIdx.x * warps + (threadIdx.x >> 5); r < n; r += (long)gridDim.x * warps) {
    const long t = r / k;
    const int p = pos[r];
    const float g = w[r];
    float dot = 0.f;
    for (int v = lane; v < vecs; v += 32) {
      float a[8], b[8], o[8];
      bb::unpack8(reinterpret_cast<const bb::bf16x8*>(dy + t * H)[v], a);
      bb::unpack8(reinterpret_cast<const bb::bf16x8*>(ys + (size_t)p * H)[v], b);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        dot += a[e] * b[e];
        o[e] = g * a[e];
      }
      reinterpret_cast<bb::bf16x8*>(dys + (size_t)p * H)[v] = bb::pack8(o);
    }
    dot = bb::warp_sum(dot);
    if (lane == 0) dw[r] = dot;
  }
}

__global__ void route_bwd_kernel(const int* __restrict__ idx, const float* __restrict__ w,
                                 const float* __restrict__ dw, float* __restrict__ dlogits, int T, int E, int k) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float s = 0.f;
  for (int j = 0; j < k; ++j) s += w[(size_t)t * k + j] * dw[(size_t)t * k + j];
  for (int j = 0; j < k; ++j) {
    const size_t r = (size_t)t * k + j;
    dlogits[(size_t)t * E + idx[r]] = w[r] * (dw[r] - s);
  }
}

}  // namespace

std::vector<torch::Tensor> moe_route(torch::Tensor logits, int64_t k) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.is_contiguous() && logits.dim() == 2,
              "moe_route: logits must be a contiguous CUDA fp32 [T, E] tensor");
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E >= 1 && E <= 32 * kMaxPerLane, "moe_route: 1 <= E <= 1024 experts");
  TORCH_CHECK(k >= 1 && k <= kMaxTopK && k <= E, "moe_route: 1 <= k <= min(32, E)");
  at::cuda::CUDAGuard guard(logits.get_device());
  auto opt_i = logits.options().dtype(at::kInt);
  auto idx = torch::empty({T, k}, opt_i);
  auto w = torch::empty({T, k}, logits.options());
  auto counts = torch::empty({E}, opt_i);
  auto offsets = torch::empty({E + 1}, opt_i);
  const long n = (long)T * k;
  auto pos = torch::empty({n}, opt_i);
  auto order = torch::empty({n}, opt_i);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (T == 0) {
    counts.zero_();
    offsets.zero_();
    return {idx, w, counts, offsets, pos, order};
  }
  {
    const int blocks = (int)std::min<long>((T + 7) / 8, 148l * 16);
    const int per = (E + 31) / 32;
#define BB_TOPK(P) topk_kernel<P><<<blocks, 256, 0, stream>>>(logits.data_ptr<float>(), T, E, (int)k, \
                                                           idx.data_ptr<int>(), w.data_ptr<float>())
    if (per <= 4) BB_TOPK(4);
    else if (per <= 8) BB_TOPK(8);
    else if (per <= 16) BB_TOPK(16);
    else BB_TOPK(32);
#undef BB_TOPK
    BB_POST_LAUNCH();
  }
  const long chunk = 4096;
  const int nb = (int)((n + chunk - 1) / chunk);
  auto block_counts = torch::empty({nb, E}, opt_i);
  block_hist_kernel<<<nb, 256, E * sizeof(int), stream>>>(idx.data_ptr<int>(), n, E, chunk,
                                                           block_counts.data_ptr<int>());
  BB_POST_LAUNCH();
  scan_kernel<<<1, 1024, 0, stream>>>(block_counts.data_ptr<int>(), nb, E, counts.data_ptr<int>(),
                                      offsets.data_ptr<int>());
  BB_POST_LAUNCH();
  place_kernel<<<nb, 256, E * sizeof(int), stream>>>(idx.data_ptr<int>(), n, E, chunk, block_counts.data_ptr<int>(),
                                                      pos.data_ptr<int>(), order.data_ptr<int>());
  BB_POST_LAUNCH();
  return {idx, w, counts, offsets, pos, order};
}

torch::Tensor moe_combine(torch::Tensor ys, torch::Tensor pos, torch::Tensor w, int64_t T) {
  TORCH_CHECK(ys.is_cuda() && ys.scalar_type() == at::kBFloat16 && ys.is_contiguous() && ys.dim() == 2,
              "moe_combine: ys must be contiguous bf16 [N, H]");
  const int H = ys.size(1);
  TORCH_CHECK(H % 8 == 0, "moe_combine: H must be a multiple of 8");
  TORCH_CHECK(pos.scalar_type() == at::kInt && w.scalar_type() == at::kFloat && pos.numel() == w.numel() &&
                  pos.is_contiguous() && w.is_contiguous() && (T == 0 || pos.numel() % T == 0),
              "moe_combine: pos (int32) and w (fp32) of T * k entries");
  auto y = torch::empty({T, H}, ys.options());
  if (T == 0) return y;
  const int k = pos.numel() / T;
  const int blocks = (int)std::min<long>((T + 7) / 8, 148l * 16);
  combine_fwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)ys.data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(),
      (int)T, H, k);
  BB_POST_LAUNCH();
  return y;
}

std::vector<torch::Tensor> moe_combine_bwd(torch::Tensor dy, torch::Tensor ys, torch::Tensor pos, torch::Tensor w) {
  TORCH_CHECK(dy.is_contiguous() && dy.scalar_type() == at::kBFloat16 && ys.is_contiguous() &&
                  dy.size(1) == ys.size(1), "moe_combine_bwd: contiguous bf16 dy [T, H] and ys [N, H]");
  const long n = pos.numel();
  const int T = dy.size(0), H = dy.size(1);
  TORCH_CHECK(T == 0 || n % T == 0, "moe_combine_bwd: pos holds T * k entries");
  auto dys = torch::empty_like(ys);   // pos is a permutation: every row is written
  auto dw = torch::empty_like(w);
  if (n == 0) return {dys, dw};
  const int k = n / T;
  const int blocks = (int)std::min<long>((n + 7) / 8, 148l * 16);
  combine_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)ys.data_ptr(), pos.data_ptr<int>(),
      w.data_ptr<float>(), (__nv_bfloat16*)dys.data_ptr(), dw.data_ptr<float>(), n, H, k);
  BB_POST_LAUNCH();
  return {dys, dw};
}

torch::Tensor moe_route_bwd(torch::Tensor idx, torch::Tensor w, torch::Tensor dw, int64_t E) {
  TORCH_CHECK(idx.is_contiguous() && w.is_contiguous() && dw.is_contiguous() && idx.dim() == 2,
              "moe_route_bwd: contiguous idx / w / dw [T, k]");
  const int T = idx.size(0), k = idx.size(1);
  auto dl = torch::zeros({T, E}, w.options());
  if (T == 0) return dl;
  route_bwd_kernel<<<(T + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int>(), w.data_ptr<float>(), dw.data_ptr<float>(), dl.data_ptr<float>(), T, (int)E, k);
  BB_POST_LAUNCH();
  return dl;
}
