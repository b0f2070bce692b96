// Gated DeltaNet element-wise kernels (forward and backward), one warp per row of D <= 256 elements:
//   gated_rmsnorm   y = RMSNorm(o) * w * silu(z)           (output gate of the GDN layer)
//   l2norm          y = x * rsqrt(sum(x^2) + eps)          (q / k normalisation before the delta rule)
//   gdn_gates       g = -exp(A_log[h]) * softplus(a + dt_bias[h]),  beta = sigmoid(b)
// FP32 math, bf16 activations; parameter gradients are reduced per block then with FP32 atomics.
// Inputs that are column slices of a fused projection ([T, H, D] views with a token stride wider
// than H * D) are read in place; outputs are contiguous.
//
// Parity: the Qwen3-Next gating / prep / gated-norm path that verl/models/mcore/tpr/gated_delta_net.py:
// 102-161 calls (MindSpeed _prepare_qkv_for_gated_delta_rule, _compute_g_and_beta, _apply_gated_norm).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace {

// Row r of a [T, H, D] view whose token stride is `st` (head stride D, unit element stride).
struct RowMap {
  long st;
  int H;
  // rows < 2^31 (checked on the host): 32-bit division
  __device__ __forceinline__ long off(long r, int D) const {
    const int ri = (int)r, t = ri / H;
    return (long)t * st + (long)(ri - t * H) * D;
  }
};

template <int E>
__device__ __forceinline__ void ld_row(const __nv_bfloat16* p, int lane, float* f) {
#pragma unroll
  for (int j = 0; j < E; ++j) f[j] = __bfloat162float(p[lane + 32 * j]);
}

template <int E>
__global__ void gated_rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ z,
                                         RowMap zm, const __nv_bfloat16* __restrict__ w,
                                         __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, long rows,
                                         float eps) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  float wv[E];
  ld_row<E>(w, lane, wv);
  for (long r = (long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long)gridDim.x * warps) {
    float x[E], g[E];
    ld_row<E>(o + r * D, lane, x);
    ld_row<E>(z + zm.off(r, D), lane, g);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) ss += x[j] * x[j];
    const float rs = rsqrtf(bb::warp_sum(ss) / D + eps);
    if (lane == 0) rstd[r] = rs;
#pragma unroll
    for (int j = 0; j < E; ++j) y[r * D + lane + 32 * j] = __float2bfloat16(x[j] * rs * wv[j] * bb::silu(g[j]));
  }
}

template <int E>
__global__ void gated_rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ o,
                                         const __nv_bfloat16* __restrict__ z, RowMap zm,
                                         const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                         __nv_bfloat16* __restrict__ d_o, __nv_bfloat16* __restrict__ dz,
                                         float* __restrict__ dw, long rows) {
  constexpr int D = 32 * E;
  __shared__ float sdw[D];
  for (int i = threadIdx.x; i < D; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  float wv[E], acc[E];
  ld_row<E>(w, lane, wv);
#pragma unroll
  for (int j = 0; j < E; ++j) acc[j] = 0.f;
  for (long r = (long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long)gridDim.x * warps) {
    float x[E], g[E], d[E];
    ld_row<E>(o + r * D, lane, x);
    ld_row<E>(z + zm.off(r, D), lane, g);
    ld_row<E>(dy + r * D, lane, d);
    const float rs = rstd[r];
    float dot = 0.f, dn[E], n[E];
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const float sg = bb::sigmoidf_(g[j]), s = g[j] * sg;
      n[j] = x[j] * rs;
      dn[j] = d[j] * wv[j] * s;
      acc[j] += d[j] * n[j] * s;
      dz[r * D + lane + 32 * j] = __float2bfloat16(d[j] * n[j] * wv[j] * sg * (1.f + g[j] * (1.f - sg)));
      dot += dn[j] * n[j];
    }
    dot = bb::warp_sum(dot) / D;
#pragma unroll
    for (int j = 0; j < E; ++j) d_o[r * D + lane + 32 * j] = __float2bfloat16(rs * (dn[j] - n[j] * dot));
  }
#pragma unroll
  for (int j = 0; j < E; ++j) atomicAdd(&sdw[lane + 32 * j], acc[j]);
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

template <int E>
__global__ void l2norm_fwd_kernel(const __nv_bfloat16* __restrict__ x, RowMap xm, __nv_bfloat16* __restrict__ y,
                                  float* __restrict__ rnorm, long rows, float eps) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (long r = (long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long)gridDim.x * warps) {
    float v[E];
    ld_row<E>(x + xm.off(r, D), lane, v);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) ss += v[j] * v[j];
    const float rs = rsqrtf(bb::warp_sum(ss) + eps);
    if (lane == 0) rnorm[r] = rs;
#pragma unroll
    for (int j = 0; j < E; ++j) y[r * D + lane + 32 * j] = __float2bfloat16(v[j] * rs);
  }
}

template <int E>
__global__ void l2norm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                  RowMap xm, const float* __restrict__ rnorm, __nv_bfloat16* __restrict__ dx,
                                  long rows) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (long r = (long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long)gridDim.x * warps) {
    float v[E], d[E];
    ld_row<E>(x + xm.off(r, D), lane, v);
    ld_row<E>(dy + r * D, lane, d);
    const float rs = rnorm[r];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) dot += d[j] * v[j] * rs;
    dot = bb::warp_sum(dot);
#pragma unroll
    for (int j = 0; j < E; ++j) dx[r * D + lane + 32 * j] = __float2bfloat16(rs * (d[j] - v[j] * rs * dot));
  }
}

__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// a, b: [T, H] with row stride lda / ldb (columns of the fused projection); g, beta: [T, H] fp32
__global__ void gdn_gates_fwd_kernel(const __nv_bfloat16* __restrict__ a, long lda, const __nv_bfloat16* __restrict__ b,
                                     long ldb, const float* __restrict__ A_log, const float* __restrict__ dt,
                                     float* __restrict__ g, float* __restrict__ beta, long T, int H) {
  const long n = T * H;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int t = (int)i / H, h = (int)i - t * H;  // n < 2^31 (host check)
    const float av = __bfloat162float(a[(long)t * lda + h]), bv = __bfloat162float(b[(long)t * ldb + h]);
    g[i] = -__expf(A_log[h]) * softplus_f(av + dt[h]);
    beta[i] = bb::sigmoidf_(bv);
  }
}

__global__ void gdn_gates_bwd_kernel(const float* __restrict__ dg, const float* __restrict__ dbeta,
                                     const __nv_bfloat16* __restrict__ a, long lda, const __nv_bfloat16* __restrict__ b,
                                     long ldb, const float* __restrict__ A_log, const float* __restrict__ dt,
                                     __nv_bfloat16* __restrict__ da, __nv_bfloat16* __restrict__ db,
                                     float* __restrict__ dA_log, float* __restrict__ ddt, long T, int H) {
  extern __shared__ float sacc[];  // [2H]: d dt_bias, d A_log partial sums of this block
  for (int i = threadIdx.x; i < 2 * H; i += blockDim.x) sacc[i] = 0.f;
  __syncthreads();
  const long n = T * H;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int t = (int)i / H, h = (int)i - t * H;  // n < 2^31 (host check)
    const float av = __bfloat162float(a[(long)t * lda + h]), bv = __bfloat162float(b[(long)t * ldb + h]);
    const float x = av + dt[h], e = __expf(A_log[h]);
    const float sp = softplus_f(x), sg = bb::sigmoidf_(x);
    const float d = dg[i];
    const float dx = -d * e * sg;  // d g / d (a + dt_bias)
    da[i] = __float2bfloat16(dx);
    atomicAdd(&sacc[h], dx);
    atomicAdd(&sacc[H + h], -d * e * sp);  // d g / d A_log = g
    const float sb = bb::sigmoidf_(bv);
    db[i] = __float2bfloat16(dbeta[i] * sb * (1.f - sb));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    atomicAdd(&ddt[i], sacc[i]);
    atomicAdd(&dA_log[i], sacc[H + i]);
  }
}

void check_rows(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name, ": contiguous CUDA bf16");
}

// [T, H, D] bf16 view with contiguous heads (strides (st, D, 1)).
RowMap row_map(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3, name, ": CUDA bf16 [T, H, D]");
  const long D = t.size(2), H = t.size(1);
  TORCH_CHECK(t.stride(2) == 1 && (H == 1 || t.stride(1) == D), name, ": heads must be contiguous rows");
  TORCH_CHECK(t.size(0) * H < (1l << 31), name, ": too many rows");
  return RowMap{t.size(0) > 1 ? t.stride(0) : H * D, (int)H};
}

}  // namespace

#define BB_ROWS_DISPATCH(D, MACRO)                                                        \
  if (D == 32) {                                                                          \
    MACRO(1);                                                                             \
  } else if (D == 64) {                                                                   \
    MACRO(2);                                                                             \
  } else if (D == 128) {                                                                  \
    MACRO(4);                                                                             \
  } else if (D == 256) {                                                                  \
    MACRO(8);                                                                             \
  } else {                                                                                \
    TORCH_CHECK(false, "GDN element-wise kernels: row width must be 32, 64, 128 or 256"); \
  }

// o: contiguous [T, H, D]; z: [T, H, D] view with contiguous heads
std::vector<torch::Tensor> gated_rmsnorm_fwd(torch::Tensor o, torch::Tensor z, torch::Tensor w, double eps) {
  check_rows(o, "o");
  const RowMap zm = row_map(z, "z");
  TORCH_CHECK(o.dim() == 3 && o.sizes() == z.sizes(), "gated_rmsnorm: o and z must be [T, H, D]");
  const int D = o.size(-1);
  const long rows = o.numel() / D;
  auto y = torch::empty_like(o);
  auto rstd = torch::empty({rows}, o.options().dtype(at::kFloat));
  if (rows == 0) return {y, rstd};
  auto wb = w.to(at::kBFloat16).contiguous();
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_GRF(E)                                                                                       \
  const int blocks = bb::resident_grid(gated_rmsnorm_fwd_kernel<E>, 256, 0, (rows + 7) / 8);                            \
  gated_rmsnorm_fwd_kernel<E><<<blocks, 256, 0, stream>>>(                                              \
      (const __nv_bfloat16*)o.data_ptr(), (const __nv_bfloat16*)z.data_ptr(), zm,                       \
      (const __nv_bfloat16*)wb.data_ptr(), (__nv_bfloat16*)y.data_ptr(), rstd.data_ptr<float>(), rows, \
      (float)eps)
  BB_ROWS_DISPATCH(D, BB_GRF)
#undef BB_GRF
  BB_POST_LAUNCH();
  return {y, rstd};
}

std::vector<torch::Tensor> gated_rmsnorm_bwd(torch::Tensor dy, torch::Tensor o, torch::Tensor z, torch::Tensor w,
                                             torch::Tensor rstd) {
  check_rows(dy, "dy");
  check_rows(o, "o");
  const RowMap zm = row_map(z, "z");
  const int D = o.size(-1);
  const long rows = o.numel() / D;
  auto d_o = torch::empty_like(o), dz = torch::empty(o.sizes(), o.options());
  auto dw = torch::zeros({D}, o.options().dtype(at::kFloat));
  if (rows == 0) return {d_o, dz, dw};
  auto wb = w.to(at::kBFloat16).contiguous();
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_GRB(E)                                                                                           \
  const int blocks = bb::resident_grid(gated_rmsnorm_bwd_kernel<E>, 256, 0, (rows + 7) / 8);                            \
  gated_rmsnorm_bwd_kernel<E><<<blocks, 256, 0, stream>>>(                                                  \
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)o.data_ptr(),                              \
      (const __nv_bfloat16*)z.data_ptr(), zm, (const __nv_bfloat16*)wb.data_ptr(), rstd.data_ptr<float>(), \
      (__nv_bfloat16*)d_o.data_ptr(), (__nv_bfloat16*)dz.data_ptr(), dw.data_ptr<float>(), rows)
  BB_ROWS_DISPATCH(D, BB_GRB)
#undef BB_GRB
  BB_POST_LAUNCH();
  return {d_o, dz, dw};
}

// x: [T, H, D] view with contiguous heads; y contiguous
std::vector<torch::Tensor> l2norm_fwd(torch::Tensor x, double eps) {
  const RowMap xm = row_map(x, "x");
  const int D = x.size(-1);
  const long rows = x.numel() / D;
  auto y = torch::empty(x.sizes(), x.options());
  auto rn = torch::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, rn};
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_L2F(E)                                                                                          \
  const int blocks = bb::resident_grid(l2norm_fwd_kernel<E>, 256, 0, (rows + 7) / 8);                            \
  l2norm_fwd_kernel<E><<<blocks, 256, 0, stream>>>((const __nv_bfloat16*)x.data_ptr(), xm,                 \
                                                   (__nv_bfloat16*)y.data_ptr(), rn.data_ptr<float>(), rows, \
                                                   (float)eps)
  BB_ROWS_DISPATCH(D, BB_L2F)
#undef BB_L2F
  BB_POST_LAUNCH();
  return {y, rn};
}

torch::Tensor l2norm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor rn) {
  check_rows(dy, "dy");
  const RowMap xm = row_map(x, "x");
  const int D = x.size(-1);
  const long rows = x.numel() / D;
  auto dx = torch::empty(x.sizes(), x.options());
  if (rows == 0) return dx;
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_L2B(E)                                                                                             \
  const int blocks = bb::resident_grid(l2norm_bwd_kernel<E>, 256, 0, (rows + 7) / 8);                            \
  l2norm_bwd_kernel<E><<<blocks, 256, 0, stream>>>((const __nv_bfloat16*)dy.data_ptr(),                        \
                                                   (const __nv_bfloat16*)x.data_ptr(), xm, rn.data_ptr<float>(), \
                                                   (__nv_bfloat16*)dx.data_ptr(), rows)
  BB_ROWS_DISPATCH(D, BB_L2B)
#undef BB_L2B
  BB_POST_LAUNCH();
  return dx;
}

// a, b: [T, H] bf16 views with unit column stride (row strides free)
std::vector<torch::Tensor> gdn_gates_fwd(torch::Tensor a, torch::Tensor b, torch::Tensor A_log, torch::Tensor dt) {
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 &&
                  a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.sizes() == b.sizes(),
              "gdn_gates: a, b must be bf16 [T, H] with contiguous columns");
  const long T = a.size(0);
  const int H = a.size(1);
  TORCH_CHECK(T * H < (1l << 31), "gdn_gates: too many elements");
  auto g = torch::empty({T, H}, a.options().dtype(at::kFloat));
  auto beta = torch::empty({T, H}, a.options().dtype(at::kFloat));
  if (T == 0) return {g, beta};
  auto Af = A_log.to(at::kFloat).contiguous(), dtf = dt.to(at::kFloat).contiguous();
  const int blocks = bb::resident_grid(gdn_gates_fwd_kernel, 256, 0, (T * H + 255) / 256);
  gdn_gates_fwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)a.data_ptr(), a.stride(0), (const __nv_bfloat16*)b.data_ptr(), b.stride(0),
      Af.data_ptr<float>(), dtf.data_ptr<float>(), g.data_ptr<float>(), beta.data_ptr<float>(), T, H);
  BB_POST_LAUNCH();
  return {g, beta};
}

std::vector<torch::Tensor> gdn_gates_bwd(torch::Tensor dg, torch::Tensor dbeta, torch::Tensor a, torch::Tensor b,
                                         torch::Tensor A_log, torch::Tensor dt) {
  const long T = a.size(0);
  const int H = a.size(1);
  TORCH_CHECK(T * H < (1l << 31), "gdn_gates: too many elements");
  auto da = torch::empty({T, H}, a.options());
  auto db = torch::empty({T, H}, a.options());
  auto dA = torch::zeros({H}, a.options().dtype(at::kFloat));
  auto ddt = torch::zeros({H}, a.options().dtype(at::kFloat));
  if (T == 0) return {da, db, dA, ddt};
  auto Af = A_log.to(at::kFloat).contiguous(), dtf = dt.to(at::kFloat).contiguous();
  auto dgc = dg.to(at::kFloat).contiguous(), dbc = dbeta.to(at::kFloat).contiguous();
  const size_t smem = 2 * H * sizeof(float);
  const int blocks = bb::resident_grid(gdn_gates_bwd_kernel, 256, smem, (T * H + 255) / 256);
  gdn_gates_bwd_kernel<<<blocks, 256, smem, at::cuda::getCurrentCUDAStream()>>>(
      dgc.data_ptr<float>(), dbc.data_ptr<float>(), (const __nv_bfloat16*)a.data_ptr(), a.stride(0),
      (const __nv_bfloat16*)b.data_ptr(), b.stride(0), Af.data_ptr<float>(), dtf.data_ptr<float>(),
      (__nv_bfloat16*)da.data_ptr(), (__nv_bfloat16*)db.data_ptr(), dA.data_ptr<float>(), ddt.data_ptr<float>(), T, H);
  BB_POST_LAUNCH();
  return {da, db, dA, ddt};
}
