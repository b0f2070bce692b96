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

#include <cstdlib>

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

// Backward, streaming form: two channels per thread (bf16x2 loads / stores, 128 bytes per warp per
// row) and one pass over the chunk's rows that reads each x and dy row once.  Registers hold a
// sliding window of the last W inputs (for the pre-activation and the weight gradient) and of the
// last W pre-activation gradients da (for dx).  dx of row p needs da(p .. p + W - 1), so the pass
// runs W - 1 rows past the chunk end; the first W - 1 da values of the sequence are kept for dh0.
template <int W>
__global__ void conv_bwd2_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                 const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias,
                                 const __nv_bfloat16* __restrict__ h0, const __nv_bfloat16* __restrict__ dhT,
                                 const int* __restrict__ cu, __nv_bfloat16* __restrict__ dx, float* __restrict__ dw,
                                 float* __restrict__ db, float* __restrict__ dh0, int C, bool silu_act) {
  const int c = 2 * (blockIdx.x * blockDim.x + threadIdx.x);   // channels c, c + 1
  const int b = blockIdx.y;
  const int q0 = cu[b], L = cu[b + 1] - q0;
  const int t0 = blockIdx.z * CH;
  if (c >= C || t0 >= L) return;
  const int t1 = min(L, t0 + CH);
  float wt[2][W];
#pragma unroll
  for (int j = 0; j < W; ++j) {
    wt[0][j] = __bfloat162float(w[(size_t)c * W + j]);
    wt[1][j] = __bfloat162float(w[(size_t)(c + 1) * W + j]);
  }
  const float bv0 = bias ? __bfloat162float(bias[c]) : 0.f, bv1 = bias ? __bfloat162float(bias[c + 1]) : 0.f;
  auto load2 = [&](const __nv_bfloat16* base, int row, float& a, float& b2) {
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(base + (size_t)(q0 + row) * C + c);
    a = __low2float(v);
    b2 = __high2float(v);
  };
  auto x_at = [&](int p, float& a, float& b2) {
    if (p >= 0) {
      load2(x, p, a, b2);
    } else if (h0) {
      a = __bfloat162float(h0[((size_t)b * C + c) * W + (W + p)]);
      b2 = __bfloat162float(h0[((size_t)b * C + c + 1) * W + (W + p)]);
    } else {
      a = b2 = 0.f;
    }
  };
  float xw[2][W];      // xw[.][W-1] = input of the current row t
  float daw[2][W];     // daw[.][W-1] = da of the current row t
#pragma unroll
  for (int j = 0; j < W; ++j) {
    daw[0][j] = daw[1][j] = 0.f;
    xw[0][j] = xw[1][j] = 0.f;
  }
#pragma unroll
  for (int j = 1; j < W; ++j) x_at(t0 - W + j, xw[0][j], xw[1][j]);   // inputs t0-W+1 .. t0-1 (slots 1..W-1)
  float gw[2][W], gb[2] = {0.f, 0.f}, head[2][W];
#pragma unroll
  for (int j = 0; j < W; ++j) gw[0][j] = gw[1][j] = head[0][j] = head[1][j] = 0.f;
  const int t_end = min(L, t1 + W - 1);
  for (int t = t0; t < t_end; ++t) {
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      xw[0][j] = xw[0][j + 1];
      xw[1][j] = xw[1][j + 1];
      daw[0][j] = daw[0][j + 1];
      daw[1][j] = daw[1][j + 1];
    }
    load2(x, t, xw[0][W - 1], xw[1][W - 1]);
    float g0, g1;
    load2(dy, t, g0, g1);
    float a0 = bv0, a1 = bv1;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      a0 += wt[0][j] * xw[0][j];
      a1 += wt[1][j] * xw[1][j];
    }
    if (silu_act) {
      const float s0 = 1.f / (1.f + __expf(-a0)), s1 = 1.f / (1.f + __expf(-a1));
      g0 *= s0 * (1.f + a0 * (1.f - s0));
      g1 *= s1 * (1.f + a1 * (1.f - s1));
    }
    daw[0][W - 1] = g0;
    daw[1][W - 1] = g1;
    if (t < t1) {                                  // weight / bias gradients of this chunk's outputs
      gb[0] += g0;
      gb[1] += g1;
#pragma unroll
      for (int j = 0; j < W; ++j) {
        gw[0][j] += g0 * xw[0][j];
        gw[1][j] += g1 * xw[1][j];
      }
      if (t < W - 1) {                             // first outputs of the sequence: they read h0
        head[0][t] = g0;
        head[1][t] = g1;
      }
    }
    const int p = t - (W - 1);                     // dx row whose da window is now complete
    if (p >= t0) {
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int j = 0; j < W; ++j) {                 // output p + W - 1 - j reads input p through tap j
        d0 += wt[0][j] * daw[0][W - 1 - j];
        d1 += wt[1][j] * daw[1][W - 1 - j];
      }
      const int sl = p - L + W;                    // final-state slot holding input p
      if (dhT && sl >= 1 && sl < W) {
        d0 += __bfloat162float(dhT[((size_t)b * C + c) * W + sl]);
        d1 += __bfloat162float(dhT[((size_t)b * C + c + 1) * W + sl]);
      }
      *reinterpret_cast<__nv_bfloat162*>(dx + (size_t)(q0 + p) * C + c) = __floats2bfloat162_rn(d0, d1);
    }
  }
  // rows of the chunk whose da window reaches past the sequence end (p > L - W): finish them with da = 0
  for (int p = t_end - (W - 1); p < t1; ++p) {   // the window shifts once per row, emitted from t0 on
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      daw[0][j] = daw[0][j + 1];
      daw[1][j] = daw[1][j + 1];
    }
    daw[0][W - 1] = daw[1][W - 1] = 0.f;
    if (p < t0) continue;
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      d0 += wt[0][j] * daw[0][W - 1 - j];
      d1 += wt[1][j] * daw[1][W - 1 - j];
    }
    const int sl = p - L + W;
    if (dhT && sl >= 1 && sl < W) {
      d0 += __bfloat162float(dhT[((size_t)b * C + c) * W + sl]);
      d1 += __bfloat162float(dhT[((size_t)b * C + c + 1) * W + sl]);
    }
    *reinterpret_cast<__nv_bfloat162*>(dx + (size_t)(q0 + p) * C + c) = __floats2bfloat162_rn(d0, d1);
  }
#pragma unroll
  for (int j = 0; j < W; ++j) {
    atomicAdd(&dw[(size_t)c * W + j], gw[0][j]);
    atomicAdd(&dw[(size_t)(c + 1) * W + j], gw[1][j]);
  }
  if (db) {
    atomicAdd(&db[c], gb[0]);
    atomicAdd(&db[c + 1], gb[1]);
  }
  if (blockIdx.z == 0 && dh0) {
    // initial-state slot s (input position s - W) is read by outputs t = 0 .. s - 1 through tap s - 1 - t
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float* hs = dh0 + ((size_t)b * C + c + q) * W;
      hs[0] = 0.f;
#pragma unroll
      for (int sidx = 1; sidx < W; ++sidx) {
        float g = 0.f;
        for (int t = 0; t < min(L, sidx); ++t) g += wt[q][sidx - 1 - t] * head[q][t];
        const int s2 = sidx - L;                   // a sequence shorter than W - 1: the final state reads it
        if (dhT && s2 >= 1) g += __bfloat162float(dhT[((size_t)b * C + c + q) * W + s2]);
        hs[sidx] = g;
      }
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
  const bool pair = (C % 2) == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) % 4) == 0 &&
                    (reinterpret_cast<uintptr_t>(dyc.data_ptr()) % 4) == 0 && !std::getenv("BB_CONV_BWD_V1");
  dim3 grid(pair ? (C / 2 + 127) / 128 : (C + 127) / 128, B, (max_len + CH - 1) / CH);
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_CB(WW)                                                                                              \
  (pair ? conv_bwd2_kernel<WW> : conv_bwd_kernel<WW>)<<<grid, 128, 0, stream>>>(                                                               \
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
