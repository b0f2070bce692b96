// Stateful causal depthwise conv1d (+ SiLU) for Gated DeltaNet, forward and backward, varlen.
//
// x [T, C] (bf16), weight [C, W], state [B, C, W] with slots 1..W-1 = the W-1 inputs before the
// sequence (slot 0 unused, always 0).  Output row t of sequence b uses inputs t-W+1..t; negative
// positions read the initial state (position p < 0 <-> slot W + p).
//
// One thread per channel, a block of 128 channels x one 64-token chunk of one sequence; reads are
// coalesced across channels.  Backward recomputes the pre-activation, produces dx, dh0 (initial
// state), consumes dhT (gradient of the final state), and accumulates dweight / dbias in FP32 with one
// atomic per (channel, tap, chunk).
//
// Parity: MindSpeed-Ops causal_conv1d with initial/final states as called from
// verl/models/mcore/tpr/gated_delta_net.py:214-236 (dh0 only for t < W-1, compact store guard).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace {

constexpr int CH = 64;

template <int W>
__device__ __forceinline__ float in_at(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ h0,
                                       int q0, int p, int c, int C, int b) {
  if (p >= 0) return __bfloat162float(x[(size_t)(q0 + p) * C + c]);
  return h0 ? __bfloat162float(h0[((size_t)b * C + c) * W + (W + p)]) : 0.f;
}

template <int W>
__global__ void conv_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ h0,
                                const int* __restrict__ cu, __nv_bfloat16* __restrict__ y,
                                __nv_bfloat16* __restrict__ hT, int C, bool silu_act) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  const int q0 = cu[b], L = cu[b + 1] - q0;
  const int t0 = blockIdx.z * CH;
  if (c >= C || t0 >= L) return;
  const int t1 = min(L, t0 + CH);
  float wt[W];
#pragma unroll
  for (int j = 0; j < W; ++j) wt[j] = __bfloat162float(w[(size_t)c * W + j]);
  const float bv = bias ? __bfloat162float(bias[c]) : 0.f;
  float win[W];  // win[W-1] = newest
#pragma unroll
  for (int j = 0; j < W - 1; ++j) win[j + 1] = in_at<W>(x, h0, q0, t0 - (W - 1) + j, c, C, b);
  for (int t = t0; t < t1; ++t) {
#pragma unroll
    for (int j = 0; j < W - 1; ++j) win[j] = win[j + 1];
    win[W - 1] = __bfloat162float(x[(size_t)(q0 + t) * C + c]);
    float a = bv;
#pragma unroll
    for (int j = 0; j < W; ++j) a += wt[j] * win[j];
    y[(size_t)(q0 + t) * C + c] = __float2bfloat16(silu_act ? bb::silu(a) : a);
  }
  if (t1 == L) {  // this chunk ends the sequence: write the final state (last W-1 inputs)
    __nv_bfloat16* hs = hT + ((size_t)b * C + c) * W;
    hs[0] = __float2bfloat16(0.f);
#pragma unroll
    for (int s = 1; s < W; ++s) hs[s] = __float2bfloat16(in_at<W>(x, h0, q0, L - W + s, c, C, b));
  }
}

template <int W>
__device__ __forceinline__ float da_at(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ h0,
                                       const __nv_bfloat16* __restrict__ dy, const float* wt, float bv, int q0, int L,
                                       int t, int c, int C, int b, bool silu_act) {
  if (t < 0 || t >= L) return 0.f;
  const float g = __bfloat162float(dy[(size_t)(q0 + t) * C + c]);
  if (!silu_act) return g;
  float a = bv;
#pragma unroll
  for (int j = 0; j < W; ++j) a += wt[j] * in_at<W>(x, h0, q0, t - (W - 1) + j, c, C, b);
  const float s = 1.f / (1.f + __expf(-a));
  return g * s * (1.f + a * (1.f - s));
}

template <int W>
__global__ void conv_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias,
                                const __nv_bfloat16* __restrict__ h0, const __nv_bfloat16* __restrict__ dhT,
                                const int* __restrict__ cu, __nv_bfloat16* __restrict__ dx, float* __restrict__ dw,
                                float* __restrict__ db, float* __restrict__ dh0, int C, bool silu_act) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  const int q0 = cu[b], L = cu[b + 1] - q0;
  const int t0 = blockIdx.z * CH;
  if (c >= C || t0 >= L) return;
  const int t1 = min(L, t0 + CH);
  float wt[W];
#pragma unroll
  for (int j = 0; j < W; ++j) wt[j] = __bfloat162float(w[(size_t)c * W + j]);
  const float bv = bias ? __bfloat162float(bias[c]) : 0.f;
  // da window for outputs p .. p+W-1 (sliding as p advances)
  float da[W];
#pragma unroll
  for (int j = 0; j < W; ++j) da[j] = da_at<W>(x, h0, dy, wt, bv, q0, L, t0 + j, c, C, b, silu_act);
  float gw[W] = {0.f}, gb = 0.f;
  for (int p = t0; p < t1; ++p) {
    // output t = p + (W-1) - j reads input p through tap j
    float g = 0.f;
#pragma unroll
    for (int j = 0; j < W; ++j) g += wt[j] * da[W - 1 - j];
    const int s = p - L + W;  // final-state slot holding input p (valid for s >= 1)
    if (dhT && s >= 1 && s < W) g += __bfloat162float(dhT[((size_t)b * C + c) * W + s]);
    dx[(size_t)(q0 + p) * C + c] = __float2bfloat16(g);
    // weight / bias grads for output t = p (da[0])
    const float d0 = da[0];
    gb += d0;
#pragma unroll
    for (int j = 0; j < W; ++j) gw[j] += d0 * in_at<W>(x, h0, q0, p - (W - 1) + j, c, C, b);
#pragma unroll
    for (int j = 0; j < W - 1; ++j) da[j] = da[j + 1];
    da[W - 1] = da_at<W>(x, h0, dy, wt, bv, q0, L, p + W, c, C, b, silu_act);
  }
#pragma unroll
  for (int j = 0; j < W; ++j) atomicAdd(&dw[(size_t)c * W + j], gw[j]);
  if (db) atomicAdd(&db[c], gb);
  if (blockIdx.z == 0 && dh0) {
    // initial-state slot s (input position s - W): read by outputs t = s - 1 - j (j taps), t in [0, L)
    float* hs = dh0 + ((size_t)b * C + c) * W;
    hs[0] = 0.f;
#pragma unroll
    for (int s = 1; s < W; ++s) {
      float g = 0.f;
      // output t reads position t-(W-1)+j through tap j, so position s-W is tap j = s-1-t (t in [0, s))
      for (int t = 0; t < min(L, s); ++t) g += wt[s - 1 - t] * da_at<W>(x, h0, dy, wt, bv, q0, L, t, c, C, b, silu_act);
      // final state slot s2 = L + s... reads initial slot s when the sequence is shorter than W-1
      const int s2 = s - L;
      if (dhT && s2 >= 1) g += __bfloat162float(dhT[((size_t)b * C + c) * W + s2]);
      hs[s] = g;
    }
  }
}

}  // namespace

std::vector<torch::Tensor> causal_conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                                             c10::optional<torch::Tensor> h0, torch::Tensor cu, int64_t max_len,
                                             bool silu_act) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "conv1d: x bf16 contiguous");
  const int T = x.size(0), C = x.size(1), W = w.size(1);
  const int B = cu.numel() - 1;
  auto wb = w.to(at::kBFloat16).contiguous();
  auto y = torch::empty_like(x);
  auto hT = torch::empty({B, C, W}, x.options());
  if (T == 0 || B == 0) return {y, hT};
  torch::Tensor h0b, biasb;
  if (h0.has_value()) h0b = h0->to(at::kBFloat16).contiguous();
  if (bias.has_value()) biasb = bias->to(at::kBFloat16).contiguous();
  dim3 grid((C + 127) / 128, B, (max_len + CH - 1) / CH);
  auto stream = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(W == 4 || W == 2 || W == 3, "conv1d: kernel width 2..4");
#define BB_CF(WW)                                                                                             \
  conv_fwd_kernel<WW><<<grid, 128, 0, stream>>>(                                                              \
      (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)wb.data_ptr(),                                 \
      bias.has_value() ? (const __nv_bfloat16*)biasb.data_ptr() : nullptr,                                    \
      h0.has_value() ? (const __nv_bfloat16*)h0b.data_ptr() : nullptr, cu.data_ptr<int>(),                    \
      (__nv_bfloat16*)y.data_ptr(), (__nv_bfloat16*)hT.data_ptr(), C, silu_act)
  if (W == 4) BB_CF(4);
  else if (W == 3) BB_CF(3);
  else BB_CF(2);
#undef BB_CF
  BB_POST_LAUNCH();
  return {y, hT};
}

std::vector<torch::Tensor> causal_conv1d_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                             c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> h0,
                                             c10::optional<torch::Tensor> dhT, torch::Tensor cu, int64_t max_len,
                                             bool silu_act) {
  const int T = x.size(0), C = x.size(1), W = w.size(1);
  const int B = cu.numel() - 1;
  auto wb = w.to(at::kBFloat16).contiguous();
  auto dx = torch::empty_like(x);
  auto dw = torch::zeros({C, W}, x.options().dtype(at::kFloat));
  auto db = torch::zeros({C}, x.options().dtype(at::kFloat));
  auto dh0 = torch::zeros({B, C, W}, x.options().dtype(at::kFloat));
  if (T == 0 || B == 0) return {dx, dw, db, dh0};
  torch::Tensor h0b, biasb, dhTb;
  if (h0.has_value()) h0b = h0->to(at::kBFloat16).contiguous();
  if (bias.has_value()) biasb = bias->to(at::kBFloat16).contiguous();
  if (dhT.has_value()) dhTb = dhT->to(at::kBFloat16).contiguous();
  auto dyc = dy.contiguous();
  dim3 grid((C + 127) / 128, B, (max_len + CH - 1) / CH);
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_CB(WW)                                                                                              \
  conv_bwd_kernel<WW><<<grid, 128, 0, stream>>>(                                                               \
      (const __nv_bfloat16*)dyc.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)wb.data_ptr(), \
      bias.has_value() ? (const __nv_bfloat16*)biasb.data_ptr() : nullptr,                                     \
      h0.has_value() ? (const __nv_bfloat16*)h0b.data_ptr() : nullptr,                                         \
      dhT.has_value() ? (const __nv_bfloat16*)dhTb.data_ptr() : nullptr, cu.data_ptr<int>(),                   \
      (__nv_bfloat16*)dx.data_ptr(), dw.data_ptr<float>(), bias.has_value() ? db.data_ptr<float>() : nullptr,  \
      h0.has_value() ? dh0.data_ptr<float>() : nullptr, C, silu_act)
  if (W == 4) BB_CB(4);
  else if (W == 3) BB_CB(3);
  else BB_CB(2);
#undef BB_CB
  BB_POST_LAUNCH();
  return {dx, dw, db, dh0};
}
