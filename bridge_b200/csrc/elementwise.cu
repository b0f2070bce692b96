// Memory-bound hot ops for sm_100a: RMSNorm, fused per-head qk-RMSNorm + RoPE, SwiGLU,
// vocab log-prob statistics / in-place logit gradient, PPO clip loss, fused AdamW.
//
// Every kernel reads its inputs once with 16-byte vector accesses and keeps all reductions in
// FP32.  Shapes are validated on the host; the kernels assume contiguous row-major tensors.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

using bb::bf16x8;

namespace {

// ----------------------------------------------------------------------------------------- RMSNorm
// One warp per row; lane owns the 8-element vectors i = lane + 32 a (a < MAXV), so a whole row stays
// in registers and HBM is touched once per tensor (all MAXV loads of a row are in flight together).
// RES = true fuses the residual add that precedes every decoder norm: h = bf16(x + res) is written
// out and normalised (the same rounding as a separate bf16 add).
template <int MAXV, bool RES>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ res,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y,
                                                          __nv_bfloat16* __restrict__ hout,
                                                          float* __restrict__ rstd, int rows, int H, float eps) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nv = H / 8;
  const bf16x8* wr = reinterpret_cast<const bf16x8*>(w);
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + (size_t)row * H);
    bf16x8 v[MAXV];
    bf16x8 rv[RES ? MAXV : 1];
#pragma unroll
    for (int a = 0; a < MAXV; ++a) {
      const int i = lane + a * 32;
      if (i < nv) {
        v[a] = xr[i];
        if constexpr (RES) rv[a] = reinterpret_cast<const bf16x8*>(res + (size_t)row * H)[i];
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int a = 0; a < MAXV; ++a) {
      const int i = lane + a * 32;
      if (i < nv) {
        float f[8];
        bb::unpack8(v[a], f);
        if constexpr (RES) {
          float g[8];
          bb::unpack8(rv[a], g);
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] += g[j];
          v[a] = bb::pack8(f);
          reinterpret_cast<bf16x8*>(hout + (size_t)row * H)[i] = v[a];
          bb::unpack8(v[a], f);  // normalise the rounded sum
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
      }
    }
    ss = bb::warp_sum(ss);
    const float r = rsqrtf(ss / H + eps);
    if (lane == 0) rstd[row] = r;
    bf16x8* yr = reinterpret_cast<bf16x8*>(y + (size_t)row * H);
#pragma unroll
    for (int a = 0; a < MAXV; ++a) {
      const int i = lane + a * 32;
      if (i < nv) {
        float f[8], g[8];
        bb::unpack8(v[a], f);
        bb::unpack8(wr[i], g);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
        yr[i] = bb::pack8(f);
      }
    }
  }
}

// dx = r * (dy*w - xhat * mean(dy*w*xhat)) (+ dres: the gradient that reached the residual sum
// directly).  dw: every warp accumulates its rows into a private FP32 row of shared memory (each lane
// owns fixed columns, so no atomics), the block sums its warps' rows and adds one FP32 atomic per
// column into dw (zero-initialised by the caller).
template <int MAXV, bool RES>
__global__ void __launch_bounds__(256, 2) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                             const __nv_bfloat16* __restrict__ x,
                                                             const __nv_bfloat16* __restrict__ w,
                                                             const float* __restrict__ rstd,
                                                             const __nv_bfloat16* __restrict__ dres,
                                                             __nv_bfloat16* __restrict__ dx, float* __restrict__ dw,
                                                             int rows, int H) {
  extern __shared__ __align__(16) float smem[];  // [H] weight (FP32), [warps][H] dw partials
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sw = smem;
  float* sdw = smem + H + (size_t)warp * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) sw[i] = __bfloat162float(w[i]);
  for (int i = threadIdx.x; i < warps * H; i += blockDim.x) smem[H + i] = 0.f;
  __syncthreads();
  const int nv = H / 8;
  for (int row = blockIdx.x * warps + warp; row < rows; row += gridDim.x * warps) {
    const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + (size_t)row * H);
    const bf16x8* gr = reinterpret_cast<const bf16x8*>(dy + (size_t)row * H);
    bf16x8 xv[MAXV], gv[MAXV];
#pragma unroll
    for (int a = 0; a < MAXV; ++a) {
      const int i = lane + a * 32;
      if (i < nv) {
        xv[a] = xr[i];
        gv[a] = gr[i];
      }
    }
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int a = 0; a < MAXV; ++a) {
      const int i = lane + a * 32;
      if (i < nv) {
        float f[8], g[8];
        bb::unpack8(xv[a], f);
        bb::unpack8(gv[a], g);
        float4* acc = reinterpret_cast<float4*>(sdw + i * 8);
        const float4* wv = reinterpret_cast<const float4*>(sw + i * 8);
        float4 a0 = acc[0], a1 = acc[1];
        const float4 w0 = wv[0], w1 = wv[1];
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float* ap0 = &a0.x;
        float* ap1 = &a1.x;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = f[j] * r;
          dot += g[j] * ww[j] * xh;
          (j < 4 ? ap0[j] : ap1[j - 4]) += g[j] * xh;
        }
        acc[0] = a0;
        acc[1] = a1;
      }
    }
    dot = bb::warp_sum(dot) / H;
    bf16x8* dxr = reinterpret_cast<bf16x8*>(dx + (size_t)row * H);
#pragma unroll
    for (int a = 0; a < MAXV; ++a) {
      const int i = lane + a * 32;
      if (i < nv) {
        float f[8], g[8], o[8], d[8];
        bb::unpack8(xv[a], f);
        bb::unpack8(gv[a], g);
        const float4* wv = reinterpret_cast<const float4*>(sw + i * 8);
        const float4 w0 = wv[0], w1 = wv[1];
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        if constexpr (RES) bb::unpack8(reinterpret_cast<const bf16x8*>(dres + (size_t)row * H)[i], d);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = r * (g[j] * ww[j] - f[j] * r * dot);
          if constexpr (RES) o[j] += d[j];
        }
        dxr[i] = bb::pack8(o);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float t = 0.f;
    for (int k = 0; k < warps; ++k) t += smem[H + (size_t)k * H + i];
    atomicAdd(&dw[i], t);
  }
}

// ------------------------------------------------------------------------------- qk-RMSNorm + RoPE
// One warp per (token, head); E = D/32 elements per lane (one 4-, 8- or 16-byte access). Rotate-half
// partner of lane l is lane l^16.
template <int E>
__device__ __forceinline__ void load_e(const __nv_bfloat16* p, float* f) {
  if constexpr (E == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  } else if constexpr (E == 8) {
    bb::unpack8(*reinterpret_cast<const bb::bf16x8*>(p), f);
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) f[j] = __bfloat162float(p[j]);
  }
}
template <int E>
__device__ __forceinline__ void store_e(__nv_bfloat16* p, const float* f) {
  if constexpr (E == 4) {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    h[0] = __floats2bfloat162_rn(f[0], f[1]);
    h[1] = __floats2bfloat162_rn(f[2], f[3]);
    *reinterpret_cast<uint2*>(p) = u;
  } else if constexpr (E == 8) {
    *reinterpret_cast<bb::bf16x8*>(p) = bb::pack8(f);
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) p[j] = __float2bfloat16(f[j]);
  }
}
// Packed bf16 row slice of E elements held in registers until use (half the registers of floats).
template <int E>
struct RawBf16 {
  using T = typename std::conditional<E == 8, uint4, typename std::conditional<E == 4, uint2, uint32_t>::type>::type;
};
template <int E>
__device__ __forceinline__ typename RawBf16<E>::T load_raw(const __nv_bfloat16* p) {
  return *reinterpret_cast<const typename RawBf16<E>::T*>(p);
}
template <int E>
__device__ __forceinline__ void unpack_raw(const typename RawBf16<E>::T& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < E / 2; ++j) {
    const float2 v = __bfloat1622float2(h[j]);
    f[2 * j] = v.x;
    f[2 * j + 1] = v.y;
  }
}

// E consecutive floats with the widest aligned vector loads (p aligned to 4 * E bytes, E in {2, 4, 8}).
template <int E>
__device__ __forceinline__ void load_f(const float* p, float* f) {
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int j = 0; j < E; j += 4) {
      const float4 v = *reinterpret_cast<const float4*>(p + j);
      f[j] = v.x; f[j + 1] = v.y; f[j + 2] = v.z; f[j + 3] = v.w;
    }
  } else if constexpr (E == 2) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    f[0] = v.x; f[1] = v.y;
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) f[j] = p[j];
  }
}

// Normalise + rotate one preloaded head row f (E = D / 32 elements per lane) and store it.
template <int D>
__device__ __forceinline__ void norm_rope_apply(float* f, const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                                float* __restrict__ rstd_out, const float* __restrict__ cs,
                                                const float* __restrict__ sn, float eps, int lane) {
  constexpr int E = D / 32;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < E; ++j) ss += f[j] * f[j];
  ss = bb::warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0) *rstd_out = r;
  float wv[E], cv[E], sv[E];
  load_f<E>(w + lane * E, wv);
#pragma unroll
  for (int j = 0; j < E; ++j) f[j] = f[j] * r * wv[j];
  // rotate half: first half lanes (0..15) hold x1, partner lanes hold x2 at the same offset.
  const bool lo = lane < 16;
  const int fi = (lane & 15) * E;  // frequency index of element 0
  load_f<E>(cs + fi, cv);
  load_f<E>(sn + fi, sv);
  float o[E];
#pragma unroll
  for (int j = 0; j < E; ++j) {
    float other = __shfl_xor_sync(0xffffffffu, f[j], 16);
    o[j] = lo ? (f[j] * cv[j] - other * sv[j]) : (f[j] * cv[j] + other * sv[j]);
  }
  store_e<E>(out + lane * E, o);
}

// A warp handles one token and kQKRows of its heads per iteration: all rows are loaded before any is
// reduced (kQKRows x 256 B in flight per warp for D = 128), and one 32-bit division per group maps
// the work item to (token, first head).
constexpr int kQKRows = 4;

template <int D>
__global__ void __launch_bounds__(256, D >= 256 ? 2 : 4) qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                        const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                        const float* __restrict__ cosb, const float* __restrict__ sinb,
                                        __nv_bfloat16* __restrict__ qo, __nv_bfloat16* __restrict__ ko,
                                        float* __restrict__ rq, float* __restrict__ rk, int T, int Hq, int Hk,
                                        float eps, long qts, long qhs, long kts, long khs) {
  __shared__ __align__(16) float swq[D], swk[D];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    swq[i] = __bfloat162float(qw[i]);
    swk[i] = __bfloat162float(kw[i]);
  }
  __syncthreads();
  constexpr int E = D / 32;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int HH = Hq + Hk, G = (HH + kQKRows - 1) / kQKRows;  // head groups per token
  const int total = T * G;                                  // < 2^31, checked on the host
  for (int item = blockIdx.x * warps + (threadIdx.x >> 5); item < total; item += gridDim.x * warps) {
    const int t = item / G, h0 = (item - t * G) * kQKRows;
    typename RawBf16<E>::T raw[kQKRows];
#pragma unroll
    for (int u = 0; u < kQKRows; ++u) {
      const int h = h0 + u;
      if (h < HH) {
        const __nv_bfloat16* src = h < Hq ? q + t * qts + h * qhs : k + t * kts + (h - Hq) * khs;
        raw[u] = load_raw<E>(src + lane * E);
      }
    }
    const float* cs = cosb + (size_t)t * (D / 2);
    const float* sn = sinb + (size_t)t * (D / 2);
#pragma unroll
    for (int u = 0; u < kQKRows; ++u) {
      const int h = h0 + u;
      if (h < HH) {
        float f[E];
        unpack_raw<E>(raw[u], f);
        if (h < Hq)
          norm_rope_apply<D>(f, swq, qo + ((size_t)t * Hq + h) * D, rq + (size_t)t * Hq + h, cs, sn, eps, lane);
        else
          norm_rope_apply<D>(f, swk, ko + ((size_t)t * Hk + h - Hq) * D, rk + (size_t)t * Hk + h - Hq, cs, sn,
                             eps, lane);
      }
    }
  }
}

// Backward of y = rope(rmsnorm(x) * w) for one preloaded row (dl = dy, x): un-rotate dy, then the
// RMSNorm backward; dw accumulated per lane.
template <int D>
__device__ __forceinline__ void norm_rope_apply_bwd(const float* dl, const float* x, const float* __restrict__ w,
                                                    float r, const float* __restrict__ cs,
                                                    const float* __restrict__ sn, __nv_bfloat16* __restrict__ dxp,
                                                    float* dwacc, int lane) {
  constexpr int E = D / 32;
  const bool lo = lane < 16;
  const int fi = (lane & 15) * E;
  float g[E], wv[E], cv[E], sv[E];
  load_f<E>(cs + fi, cv);
  load_f<E>(sn + fi, sv);
  load_f<E>(w + lane * E, wv);
#pragma unroll
  for (int j = 0; j < E; ++j) {
    float d = dl[j];
    float other = __shfl_xor_sync(0xffffffffu, d, 16);
    // forward: lo: y = a c - b s ; hi: y = b c + a s  (a = x1, b = x2)
    g[j] = lo ? (d * cv[j] + other * sv[j]) : (d * cv[j] - other * sv[j]);
  }
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    float xh = x[j] * r;
    dot += g[j] * wv[j] * xh;
    dwacc[j] += g[j] * xh;
  }
  dot = bb::warp_sum(dot) / D;
  float o[E];
#pragma unroll
  for (int j = 0; j < E; ++j) o[j] = r * (g[j] * wv[j] - x[j] * r * dot);
  store_e<E>(dxp + lane * E, o);
}

template <int D>
__global__ void __launch_bounds__(256, D >= 256 ? 2 : 4) qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dqo, const __nv_bfloat16* __restrict__ dko,
                                        const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                        const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                        const float* __restrict__ cosb, const float* __restrict__ sinb,
                                        const float* __restrict__ rq, const float* __restrict__ rk,
                                        __nv_bfloat16* __restrict__ dq, __nv_bfloat16* __restrict__ dk,
                                        float* __restrict__ dqw, float* __restrict__ dkw, int T, int Hq, int Hk,
                                        long qts, long qhs, long kts, long khs) {
  constexpr int E = D / 32;
  __shared__ __align__(16) float swq[D], swk[D], sdq[D], sdk[D];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    swq[i] = __bfloat162float(qw[i]);
    swk[i] = __bfloat162float(kw[i]);
    sdq[i] = 0.f;
    sdk[i] = 0.f;
  }
  __syncthreads();
  float aq[E], ak[E];
#pragma unroll
  for (int j = 0; j < E; ++j) aq[j] = ak[j] = 0.f;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int HH = Hq + Hk, G = (HH + kQKRows - 1) / kQKRows;
  const int total = T * G;
  for (int item = blockIdx.x * warps + (threadIdx.x >> 5); item < total; item += gridDim.x * warps) {
    const int t = item / G, h0 = (item - t * G) * kQKRows;
    typename RawBf16<E>::T rd[kQKRows], rx[kQKRows];
    float rr[kQKRows];
#pragma unroll
    for (int u = 0; u < kQKRows; ++u) {
      const int h = h0 + u;
      if (h < HH) {
        if (h < Hq) {
          rd[u] = load_raw<E>(dqo + ((size_t)t * Hq + h) * D + lane * E);
          rx[u] = load_raw<E>(q + t * qts + h * qhs + lane * E);
          rr[u] = rq[(size_t)t * Hq + h];
        } else {
          rd[u] = load_raw<E>(dko + ((size_t)t * Hk + h - Hq) * D + lane * E);
          rx[u] = load_raw<E>(k + t * kts + (h - Hq) * khs + lane * E);
          rr[u] = rk[(size_t)t * Hk + h - Hq];
        }
      }
    }
    const float* cs = cosb + (size_t)t * (D / 2);
    const float* sn = sinb + (size_t)t * (D / 2);
#pragma unroll
    for (int u = 0; u < kQKRows; ++u) {
      const int h = h0 + u;
      if (h < HH) {
        float dl[E], xv[E];
        unpack_raw<E>(rd[u], dl);
        unpack_raw<E>(rx[u], xv);
        if (h < Hq)
          norm_rope_apply_bwd<D>(dl, xv, swq, rr[u], cs, sn, dq + ((size_t)t * Hq + h) * D, aq, lane);
        else
          norm_rope_apply_bwd<D>(dl, xv, swk, rr[u], cs, sn, dk + ((size_t)t * Hk + h - Hq) * D, ak, lane);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < E; ++j) {
    atomicAdd(&sdq[lane * E + j], aq[j]);
    atomicAdd(&sdk[lane * E + j], ak[j]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    atomicAdd(&dqw[i], sdq[i]);
    atomicAdd(&dkw[i], sdk[i]);
  }
}

// ----------------------------------------------------------------------------------------- SwiGLU
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ y, long rows,
                                  int F) {
  const int nv = F / 8;
  const long total = rows * nv;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)i / nv, c = (int)i - r * nv;  // rows * nv < 2^31 (host check)
    const bf16x8* g = reinterpret_cast<const bf16x8*>(gu + (size_t)r * 2 * F) + c;
    const bf16x8* u = reinterpret_cast<const bf16x8*>(gu + (size_t)r * 2 * F + F) + c;
    float a[8], b[8];
    bb::unpack8(*g, a);
    bb::unpack8(*u, b);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = bb::silu(a[j]) * b[j];
    reinterpret_cast<bf16x8*>(y + (size_t)r * F)[c] = bb::pack8(a);
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, long rows, int F) {
  const int nv = F / 8;
  const long total = rows * nv;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)i / nv, c = (int)i - r * nv;  // rows * nv < 2^31 (host check)
    float a[8], b[8], d[8], da[8], db[8];
    bb::unpack8(reinterpret_cast<const bf16x8*>(gu + (size_t)r * 2 * F)[c], a);
    bb::unpack8(reinterpret_cast<const bf16x8*>(gu + (size_t)r * 2 * F + F)[c], b);
    bb::unpack8(reinterpret_cast<const bf16x8*>(dy + (size_t)r * F)[c], d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float s = bb::sigmoidf_(a[j]);
      float sl = a[j] * s;
      db[j] = d[j] * sl;
      da[j] = d[j] * b[j] * s * (1.f + a[j] * (1.f - s));
    }
    reinterpret_cast<bf16x8*>(dgu + (size_t)r * 2 * F)[c] = bb::pack8(da);
    reinterpret_cast<bf16x8*>(dgu + (size_t)r * 2 * F + F)[c] = bb::pack8(db);
  }
}

// -------------------------------------------------------------------------------- log-prob over vocab
// One block per row: online (max, sum exp, sum exp*z) of z = logit * inv_temp; target logit if local.
__global__ void logprob_stats_kernel(const __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ targets,
                                     const float* __restrict__ inv_temp, float* __restrict__ stats, int V,
                                     long vocab_start) {
  const int row = blockIdx.x;
  const float it = inv_temp[row];
  const __nv_bfloat16* lr = logits + (size_t)row * V;
  float m = -INFINITY, s = 0.f, ez = 0.f;
  auto push = [&](float z) {
    if (z > m) {
      float c = __expf(m - z);
      s *= c;
      ez *= c;
      m = z;
    }
    float e = __expf(z - m);
    s += e;
    ez += e * z;
  };
  if ((V & 7) == 0) {
    const bf16x8* v8 = reinterpret_cast<const bf16x8*>(lr);
    for (int i = threadIdx.x; i < V / 8; i += blockDim.x) {
      float f[8];
      bb::unpack8(v8[i], f);
      float bm = f[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) bm = fmaxf(bm, f[j]);
      bm *= it;
      if (bm > m) {
        float c = __expf(m - bm);
        s *= c;
        ez *= c;
        m = bm;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float z = f[j] * it;
        float e = __expf(z - m);
        s += e;
        ez += e * z;
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) push(__bfloat162float(lr[i]) * it);
  }
  // combine across the block
  __shared__ float sm[32], ss[32], se[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    float e2 = __shfl_xor_sync(0xffffffffu, ez, o);
    float mm = fmaxf(m, m2);
    float a = (m == -INFINITY) ? 0.f : __expf(m - mm), b = (m2 == -INFINITY) ? 0.f : __expf(m2 - mm);
    s = s * a + s2 * b;
    ez = ez * a + e2 * b;
    m = mm;
  }
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
    se[warp] = ez;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
    ez = lane < nw ? se[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      float e2 = __shfl_xor_sync(0xffffffffu, ez, o);
      float mm = fmaxf(m, m2);
      float a = (m == -INFINITY) ? 0.f : __expf(m - mm), b = (m2 == -INFINITY) ? 0.f : __expf(m2 - mm);
      s = s * a + s2 * b;
      ez = ez * a + e2 * b;
      m = mm;
    }
    if (lane == 0) {
      long t = targets[row] - vocab_start;
      float tz = (t >= 0 && t < V) ? __bfloat162float(lr[t]) * it : 0.f;
      stats[row * 4 + 0] = m;
      stats[row * 4 + 1] = s;
      stats[row * 4 + 2] = tz;
      stats[row * 4 + 3] = ez;
    }
  }
}

__global__ void logprob_finalize_kernel(const float* __restrict__ stats, float* __restrict__ lse,
                                        float* __restrict__ lp, float* __restrict__ ent, float* __restrict__ ezn,
                                        int U) {
  int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= U) return;
  float m = stats[u * 4], s = stats[u * 4 + 1], tz = stats[u * 4 + 2], ez = stats[u * 4 + 3];
  float l = m + __logf(s);
  lse[u] = l;
  lp[u] = tz - l;
  ezn[u] = ez / s;
  ent[u] = l - ez / s;
}

// In place: logits[u, v] <- d loss / d logits = it * (dlp*(1[v==t] - p) - dent*p*(z - Ez)),  p = exp(z - lse).
__global__ void logprob_grad_kernel(__nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ targets,
                                    const float* __restrict__ inv_temp, const float* __restrict__ lse,
                                    const float* __restrict__ ezn, const float* __restrict__ dlp,
                                    const float* __restrict__ dent, int V, long vocab_start) {
  const int row = blockIdx.x;
  const float it = inv_temp[row], l = lse[row], g = dlp[row];
  const float de = dent ? dent[row] : 0.f, e = ezn[row];
  const long t = targets[row] - vocab_start;
  __nv_bfloat16* lr = logits + (size_t)row * V;
  if ((V & 7) == 0) {
    bf16x8* v8 = reinterpret_cast<bf16x8*>(lr);
    for (int i = threadIdx.x; i < V / 8; i += blockDim.x) {
      float f[8];
      bb::unpack8(v8[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float z = f[j] * it;
        float p = __expf(z - l);
        float d = -g * p - de * p * (z - e);
        if ((long)(i * 8 + j) == t) d += g;
        f[j] = d * it;
      }
      v8[i] = bb::pack8(f);
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      float z = __bfloat162float(lr[i]) * it;
      float p = __expf(z - l);
      float d = -g * p - de * p * (z - e);
      if ((long)i == t) d += g;
      lr[i] = __float2bfloat16(d * it);
    }
  }
}

// ----------------------------------------------------------------------------------------- PPO loss
// Grid-stride over the tokens; each block writes its five partial sums (loss, clip, dual clip, -log ratio,
// ratio) to part[block]; ppo_loss_finalize_kernel sums the blocks in a fixed order (deterministic).
__global__ void ppo_loss_kernel(const float* __restrict__ x, const float* __restrict__ old,
                                const float* __restrict__ adv, const float* __restrict__ wts, float* __restrict__ part,
                                float* __restrict__ grad, long n, float inv_denom, float lo, float hi, float cdual) {
  __shared__ float scratch[32];
  float ls = 0.f, cf = 0.f, dcf = 0.f, kl = 0.f, rs = 0.f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float a = adv[i];
    const float d = x[i] - old[i];
    const float dc = fminf(fmaxf(d, -20.f), 20.f);
    const float r = __expf(dc);
    const float dr = (d > -20.f && d < 20.f) ? r : 0.f;  // d r / d x
    const float l1 = -a * r;
    const float rc = fminf(fmaxf(r, 1.f - lo), 1.f + hi);
    const float l2 = -a * rc;
    const float d1 = -a * dr;
    const float d2 = (r >= 1.f - lo && r <= 1.f + hi) ? -a * dr : 0.f;
    float prim = l1, dprim = d1;
    if (l2 > l1) {
      prim = l2;
      dprim = d2;
    }
    float loss = prim, dl = dprim;
    const float dual = -a * cdual;
    if (a < 0.f && prim > dual) {
      loss = dual;
      dl = 0.f;
    }
    const float w = wts ? wts[i] : 1.f;
    ls += loss * w;
    grad[i] = dl * w * inv_denom;
    cf += (l2 > l1) ? 1.f : 0.f;
    dcf += (a < 0.f && prim > dual) ? 1.f : 0.f;
    kl += -d;
    rs += r;
  }
  ls = bb::block_sum(ls, scratch);
  cf = bb::block_sum(cf, scratch);
  dcf = bb::block_sum(dcf, scratch);
  kl = bb::block_sum(kl, scratch);
  rs = bb::block_sum(rs, scratch);
  if (threadIdx.x == 0) {
    float* p = part + 5 * (long)blockIdx.x;
    p[0] = ls;
    p[1] = cf;
    p[2] = dcf;
    p[3] = kl;
    p[4] = rs;
  }
}

__global__ void ppo_loss_finalize_kernel(const float* __restrict__ part, int blocks, long n, float inv_denom,
                                         float* __restrict__ out, float* __restrict__ stats) {
  if (threadIdx.x != 0) return;
  float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
  for (int b = 0; b < blocks; ++b)
    for (int j = 0; j < 5; ++j) acc[j] += part[5 * b + j];
  out[0] = acc[0] * inv_denom;
  const float inv_n = 1.f / (float)(n > 0 ? n : 1);
  for (int j = 0; j < 4; ++j) stats[j] = acc[j + 1] * inv_n;
}

// ----------------------------------------------------------------------------------------- AdamW
template <typename P>
__global__ void adamw_kernel(float* __restrict__ master, P* __restrict__ param, const float* __restrict__ grad,
                             float* __restrict__ m, float* __restrict__ v, const float* __restrict__ clip, long n,
                             float lr, float b1, float b2, float eps, float wd, float bc1, float bc2, bool vec) {
  const float c = clip[0];
  const float inv_bc1 = 1.f / bc1, inv_sqrt_bc2 = rsqrtf(bc2);
  auto step = [&](float g, float& mi, float& vi, float& w) {
    g *= c;
    mi = b1 * mi + (1.f - b1) * g;
    vi = b2 * vi + (1.f - b2) * g * g;
    w = w * (1.f - lr * wd) - lr * (mi * inv_bc1) / (sqrtf(vi) * inv_sqrt_bc2 + eps);
  };
  // 16-byte vectors when every pointer allows them (decided on the host), then a scalar tail
  const long n4 = vec ? n / 4 : 0;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 g = reinterpret_cast<const float4*>(grad)[i];
    float4 mi = reinterpret_cast<float4*>(m)[i], vi = reinterpret_cast<float4*>(v)[i];
    float4 w = reinterpret_cast<float4*>(master)[i];
    step(g.x, mi.x, vi.x, w.x);
    step(g.y, mi.y, vi.y, w.y);
    step(g.z, mi.z, vi.z, w.z);
    step(g.w, mi.w, vi.w, w.w);
    reinterpret_cast<float4*>(m)[i] = mi;
    reinterpret_cast<float4*>(v)[i] = vi;
    reinterpret_cast<float4*>(master)[i] = w;
    if constexpr (std::is_same<P, float>::value) {
      reinterpret_cast<float4*>(param)[i] = w;
    } else {
      uint2 u;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
      h[0] = __floats2bfloat162_rn(w.x, w.y);
      h[1] = __floats2bfloat162_rn(w.z, w.w);
      reinterpret_cast<uint2*>(param)[i] = u;
    }
  }
  const long stride = vec ? blockDim.x : (long)gridDim.x * blockDim.x;
  const long first = vec ? (blockIdx.x == 0 ? n4 * 4 + threadIdx.x : n) : (long)blockIdx.x * blockDim.x + threadIdx.x;
  for (long i = first; i < n; i += stride) {
    float mi = m[i], vi = v[i], w = master[i];
    step(grad[i], mi, vi, w);
    m[i] = mi;
    v[i] = vi;
    master[i] = w;
    if constexpr (std::is_same<P, float>::value) {
      param[i] = w;
    } else {
      param[i] = __float2bfloat16(w);
    }
  }
}

// Sum of squares of an FP32 vector in one read: per-block partials (float4 loads, FP32 accumulation
// per thread, fixed-order block reduction), then one block sums the partials in a fixed order, so the
// result is deterministic.
__global__ void sumsq_partial_kernel(const float* __restrict__ x, long n, bool vec, float* __restrict__ part) {
  float acc = 0.f;
  const long n4 = vec ? n / 4 : 0;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(x)[i];
    acc += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  for (long i = n4 * 4 + (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    acc += x[i] * x[i];
  __shared__ float sw[32];
  acc = bb::warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sw[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sw[threadIdx.x] : 0.f;
    t = bb::warp_sum(t);
    if (threadIdx.x == 0) part[blockIdx.x] = t;
  }
}

__global__ void sum_partials_kernel(const float* __restrict__ part, int n, float* __restrict__ out, bool accumulate) {
  __shared__ float sw[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += part[i];
  acc = bb::warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sw[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sw[threadIdx.x] : 0.f;
    t = bb::warp_sum(t);
    if (threadIdx.x == 0) out[0] = accumulate ? out[0] + t : t;
  }
}

// ------------------------------------------------------------------------------------ embedding
// Vocab-parallel lookup (rows [start, start + rows) of the full table live here; other ids give zero
// rows) and its backward as a scatter-add of dy rows into the FP32 gradient buffer (16-byte float4
// atomics; repeated ids add in arbitrary order).  One warp per token, 16-byte accesses.
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ w,
                                     __nv_bfloat16* __restrict__ out, int T, int H, long start, long rows) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31, nv = H / 8;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const long r = ids[t] - start;
    const bool ok = r >= 0 && r < rows;
    bf16x8* dst = reinterpret_cast<bf16x8*>(out + (size_t)t * H);
    const bf16x8* src = reinterpret_cast<const bf16x8*>(w + (size_t)(ok ? r : 0) * H);
    for (int i = lane; i < nv; i += 32) {
      bf16x8 v;
      if (ok) {
        v = src[i];
      } else {
        float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        v = bb::pack8(z);
      }
      dst[i] = v;
    }
  }
}

__global__ void embedding_bwd_acc_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                         float* __restrict__ g, int T, int H, long start, long rows) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31, nv = H / 8;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const long r = ids[t] - start;
    if (r < 0 || r >= rows) continue;
    const bf16x8* src = reinterpret_cast<const bf16x8*>(dy + (size_t)t * H);
    float4* dst = reinterpret_cast<float4*>(g + (size_t)r * H);
    for (int i = lane; i < nv; i += 32) {
      float f[8];
      bb::unpack8(src[i], f);
      atomicAdd(dst + 2 * i, make_float4(f[0], f[1], f[2], f[3]));
      atomicAdd(dst + 2 * i + 1, make_float4(f[4], f[5], f[6], f[7]));
    }
  }
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

void check_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
              " must be a contiguous CUDA bf16 tensor");
}

}  // namespace

// ============================================================================================ host
// MAXV = ceil(H / 256) 16-byte vectors per lane (10 for H = 2560); H % 8 == 0, H <= 4096.
#define BB_RMS_DISPATCH(nv, MACRO)                                                 \
  if (nv <= 32) {                                                                  \
    MACRO(1);                                                                      \
  } else if (nv <= 64) {                                                           \
    MACRO(2);                                                                      \
  } else if (nv <= 128) {                                                          \
    MACRO(4);                                                                      \
  } else if (nv <= 192) {                                                          \
    MACRO(6);                                                                      \
  } else if (nv <= 256) {                                                          \
    MACRO(8);                                                                      \
  } else if (nv <= 320) {                                                          \
    MACRO(10);                                                                     \
  } else if (nv <= 384) {                                                          \
    MACRO(12);                                                                     \
  } else if (nv <= 512) {                                                          \
    MACRO(16);                                                                     \
  } else {                                                                         \
    TORCH_CHECK(false, "rmsnorm: hidden size above 4096 is not supported");        \
  }

namespace {
std::vector<torch::Tensor> rmsnorm_fwd_impl(torch::Tensor x, c10::optional<torch::Tensor> res, torch::Tensor w,
                                            double eps) {
  check_bf16(x, "x");
  check_bf16(w, "weight");
  const int H = x.size(-1);
  TORCH_CHECK(H % 8 == 0 && w.numel() == H, "rmsnorm: hidden must be a multiple of 8 and match weight");
  const long rows = x.numel() / H;
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  torch::Tensor h;
  if (res) {
    check_bf16(*res, "residual");
    TORCH_CHECK(res->sizes() == x.sizes(), "rmsnorm: residual shape must match x");
    h = torch::empty_like(x);
  }
  if (rows == 0) return res ? std::vector<torch::Tensor>{y, rstd, h} : std::vector<torch::Tensor>{y, rstd};
  const int threads = 256;
  const int nv = H / 8;
  auto stream = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* rp = res ? (const __nv_bfloat16*)res->data_ptr() : nullptr;
  __nv_bfloat16* hp = res ? (__nv_bfloat16*)h.data_ptr() : nullptr;
#define BB_RMS_FWD(MV)                                                                                        \
  const int blocks = res ? bb::resident_grid(rmsnorm_fwd_kernel<MV, true>, threads, 0, (rows + 7) / 8)         \
                         : bb::resident_grid(rmsnorm_fwd_kernel<MV, false>, threads, 0, (rows + 7) / 8);       \
  if (res)                                                                                                    \
    rmsnorm_fwd_kernel<MV, true><<<blocks, threads, 0, stream>>>(                                             \
        (const __nv_bfloat16*)x.data_ptr(), rp, (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(), \
        hp, rstd.data_ptr<float>(), rows, H, (float)eps);                                                     \
  else                                                                                                        \
    rmsnorm_fwd_kernel<MV, false><<<blocks, threads, 0, stream>>>(                                            \
        (const __nv_bfloat16*)x.data_ptr(), nullptr, (const __nv_bfloat16*)w.data_ptr(),                      \
        (__nv_bfloat16*)y.data_ptr(), nullptr, rstd.data_ptr<float>(), rows, H, (float)eps)
  BB_RMS_DISPATCH(nv, BB_RMS_FWD)
#undef BB_RMS_FWD
  BB_POST_LAUNCH();
  return res ? std::vector<torch::Tensor>{y, rstd, h} : std::vector<torch::Tensor>{y, rstd};
}

std::vector<torch::Tensor> rmsnorm_bwd_impl(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                                            c10::optional<torch::Tensor> dres,
                                            c10::optional<torch::Tensor> dw_acc = c10::nullopt) {
  check_bf16(dy, "dy");
  check_bf16(x, "x");
  const int H = x.size(-1);
  const long rows = x.numel() / H;
  auto dx = torch::empty_like(x);
  torch::Tensor dw;
  if (dw_acc) {  // accumulate straight into an FP32 gradient buffer (e.g. the weight's main_grad)
    TORCH_CHECK(dw_acc->is_cuda() && dw_acc->scalar_type() == at::kFloat && dw_acc->is_contiguous() &&
                    dw_acc->numel() == H, "rmsnorm_bwd: dw accumulator must be a contiguous FP32 [H] tensor");
    dw = *dw_acc;
  } else {
    dw = torch::zeros({H}, x.options().dtype(at::kFloat));
  }
  if (dres) {
    check_bf16(*dres, "dres");
    TORCH_CHECK(dres->sizes() == x.sizes(), "rmsnorm_bwd: residual gradient shape must match x");
  }
  if (rows == 0) return {dx, dw};
  const int threads = 256;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int nv = H / 8;
  const size_t smem = (1 + threads / 32) * (size_t)H * sizeof(float);
  const __nv_bfloat16* dp = dres ? (const __nv_bfloat16*)dres->data_ptr() : nullptr;
#define BB_RMS_BWD(MV)                                                                                        \
  cudaFuncSetAttribute(rmsnorm_bwd_kernel<MV, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);  \
  cudaFuncSetAttribute(rmsnorm_bwd_kernel<MV, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
  const int blocks = dres ? bb::resident_grid(rmsnorm_bwd_kernel<MV, true>, threads, smem, (rows + 7) / 8)    \
                          : bb::resident_grid(rmsnorm_bwd_kernel<MV, false>, threads, smem, (rows + 7) / 8);  \
  if (dres)                                                                                                   \
    rmsnorm_bwd_kernel<MV, true><<<blocks, threads, smem, stream>>>(                                          \
        (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), \
        rstd.data_ptr<float>(), dp, (__nv_bfloat16*)dx.data_ptr(), dw.data_ptr<float>(), rows, H);           \
  else                                                                                                        \
    rmsnorm_bwd_kernel<MV, false><<<blocks, threads, smem, stream>>>(                                         \
        (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), \
        rstd.data_ptr<float>(), nullptr, (__nv_bfloat16*)dx.data_ptr(), dw.data_ptr<float>(), rows, H)
  BB_RMS_DISPATCH(nv, BB_RMS_BWD)
#undef BB_RMS_BWD
  BB_POST_LAUNCH();
  return {dx, dw};
}
}  // namespace

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  return rmsnorm_fwd_impl(x, c10::nullopt, w, eps);
}

std::vector<torch::Tensor> rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd) {
  return rmsnorm_bwd_impl(dy, x, w, rstd, c10::nullopt);
}

// h = x + res; y = RMSNorm(h) * w  ->  {y, rstd, h}
std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor res, torch::Tensor w, double eps) {
  return rmsnorm_fwd_impl(x, res, w, eps);
}

// dx (+ dres when given, i.e. non-empty) with dw accumulated into dw_acc (FP32 [H]) -> dx
torch::Tensor rmsnorm_bwd_acc(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dres,
                              torch::Tensor dw_acc) {
  c10::optional<torch::Tensor> r = dres.numel() ? c10::optional<torch::Tensor>(dres) : c10::nullopt;
  return rmsnorm_bwd_impl(dy, x, w, rstd, r, dw_acc)[0];
}

// d(x) = d(res) = rmsnorm_bwd(dy) + dh  ->  {dsum, dw}
std::vector<torch::Tensor> add_rmsnorm_bwd(torch::Tensor dy, torch::Tensor h, torch::Tensor w, torch::Tensor rstd,
                                           torch::Tensor dh) {
  return rmsnorm_bwd_impl(dy, h, w, rstd, dh);
}

// q [T, Hq, D], k [T, Hk, D] may be strided views (e.g. column slices of a fused QKV output): the
// head dimension must be contiguous, token / head strides 16-byte aligned; outputs are contiguous.
void check_qk_view(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3 && t.stride(2) == 1 &&
                  t.stride(0) % 8 == 0 && t.stride(1) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              name, " must be a bf16 [T, H, D] view with a contiguous, 16-byte aligned head dimension");
}

std::vector<torch::Tensor> qk_norm_rope_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor qw, torch::Tensor kw,
                                            torch::Tensor cosb, torch::Tensor sinb, double eps) {
  check_qk_view(q, "q");
  check_qk_view(k, "k");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && q.size(2) == k.size(2) && q.size(0) == k.size(0), "qk shapes");
  const int T = q.size(0), Hq = q.size(1), Hk = k.size(1), D = q.size(2);
  TORCH_CHECK(cosb.size(0) == T && cosb.size(1) == D / 2 && cosb.scalar_type() == at::kFloat && cosb.is_contiguous() &&
                  sinb.is_contiguous() && (reinterpret_cast<uintptr_t>(cosb.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sinb.data_ptr()) & 15) == 0,
              "cos / sin tables must be contiguous, 16-byte aligned [T, D/2] fp32");
  auto qo = torch::empty({T, Hq, D}, q.options()), ko = torch::empty({T, Hk, D}, k.options());
  auto rq = torch::empty({T, Hq}, q.options().dtype(at::kFloat));
  auto rk = torch::empty({T, Hk}, q.options().dtype(at::kFloat));
  if (T == 0) return {qo, ko, rq, rk};
  const int threads = 256;
  const long items = (long)T * ((Hq + Hk + kQKRows - 1) / kQKRows);
  TORCH_CHECK(items < (1l << 31), "qk_norm_rope: too many rows");
  auto stream = at::cuda::getCurrentCUDAStream();
  auto qwb = qw.contiguous(), kwb = kw.contiguous();
#define BB_QKF(DD)                                                                                               \
  const int blocks = bb::resident_grid(qk_norm_rope_fwd_kernel<DD>, threads, 0, (items + 7) / 8);                 \
  qk_norm_rope_fwd_kernel<DD><<<blocks, threads, 0, stream>>>(                                                   \
      (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)qwb.data_ptr(), \
      (const __nv_bfloat16*)kwb.data_ptr(), cosb.data_ptr<float>(), sinb.data_ptr<float>(),                      \
      (__nv_bfloat16*)qo.data_ptr(), (__nv_bfloat16*)ko.data_ptr(), rq.data_ptr<float>(), rk.data_ptr<float>(), T, \
      Hq, Hk, (float)eps, q.stride(0), q.stride(1), k.stride(0), k.stride(1))
  if (D == 128) {
    BB_QKF(128);
  } else if (D == 64) {
    BB_QKF(64);
  } else if (D == 256) {
    BB_QKF(256);
  } else {
    TORCH_CHECK(false, "qk_norm_rope: head_dim must be 64, 128 or 256");
  }
#undef BB_QKF
  BB_POST_LAUNCH();
  return {qo, ko, rq, rk};
}

namespace {
std::vector<torch::Tensor> qk_norm_rope_bwd_impl(torch::Tensor dqo, torch::Tensor dko, torch::Tensor q, torch::Tensor k,
                                                 torch::Tensor qw, torch::Tensor kw, torch::Tensor cosb,
                                                 torch::Tensor sinb, torch::Tensor rq, torch::Tensor rk,
                                                 torch::Tensor dqw_acc, torch::Tensor dkw_acc) {
  check_bf16(dqo, "dq");
  check_bf16(dko, "dk");
  check_qk_view(q, "q");
  check_qk_view(k, "k");
  TORCH_CHECK(cosb.is_contiguous() && sinb.is_contiguous() && (reinterpret_cast<uintptr_t>(cosb.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sinb.data_ptr()) & 15) == 0,
              "cos / sin tables must be contiguous and 16-byte aligned");
  const int T = q.size(0), Hq = q.size(1), Hk = k.size(1), D = q.size(2);
  auto dq = torch::empty({T, Hq, D}, q.options()), dk = torch::empty({T, Hk, D}, k.options());
  auto acc_ok = [&](const torch::Tensor& t) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == D,
                "qk_norm_rope_bwd: weight-gradient accumulators must be contiguous FP32 [D] tensors");
    return t;
  };
  // empty accumulators: fresh zeroed outputs; otherwise accumulate into them (e.g. the weights' main_grad)
  auto dqw = dqw_acc.numel() ? acc_ok(dqw_acc) : torch::zeros({D}, q.options().dtype(at::kFloat));
  auto dkw = dkw_acc.numel() ? acc_ok(dkw_acc) : torch::zeros({D}, q.options().dtype(at::kFloat));
  if (T == 0) return {dq, dk, dqw, dkw};
  const int threads = 256;
  const long items = (long)T * ((Hq + Hk + kQKRows - 1) / kQKRows);
  TORCH_CHECK(items < (1l << 31), "qk_norm_rope: too many rows");
  auto stream = at::cuda::getCurrentCUDAStream();
  auto qwb = qw.contiguous(), kwb = kw.contiguous();
#define BB_QKB(DD)                                                                                               \
  const int blocks = bb::resident_grid(qk_norm_rope_bwd_kernel<DD>, threads, 0, (items + 7) / 8);                 \
  qk_norm_rope_bwd_kernel<DD><<<blocks, threads, 0, stream>>>(                                                   \
      (const __nv_bfloat16*)dqo.data_ptr(), (const __nv_bfloat16*)dko.data_ptr(), (const __nv_bfloat16*)q.data_ptr(), \
      (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)qwb.data_ptr(), (const __nv_bfloat16*)kwb.data_ptr(), \
      cosb.data_ptr<float>(), sinb.data_ptr<float>(), rq.data_ptr<float>(), rk.data_ptr<float>(),                \
      (__nv_bfloat16*)dq.data_ptr(), (__nv_bfloat16*)dk.data_ptr(), dqw.data_ptr<float>(), dkw.data_ptr<float>(), T, \
      Hq, Hk, q.stride(0), q.stride(1), k.stride(0), k.stride(1))
  if (D == 128) {
    BB_QKB(128);
  } else if (D == 64) {
    BB_QKB(64);
  } else if (D == 256) {
    BB_QKB(256);
  } else {
    TORCH_CHECK(false, "qk_norm_rope: head_dim must be 64, 128 or 256");
  }
#undef BB_QKB
  BB_POST_LAUNCH();
  return {dq, dk, dqw, dkw};
}
}  // namespace

std::vector<torch::Tensor> qk_norm_rope_bwd(torch::Tensor dqo, torch::Tensor dko, torch::Tensor q, torch::Tensor k,
                                            torch::Tensor qw, torch::Tensor kw, torch::Tensor cosb,
                                            torch::Tensor sinb, torch::Tensor rq, torch::Tensor rk) {
  auto none = torch::empty({0}, q.options().dtype(at::kFloat));
  return qk_norm_rope_bwd_impl(dqo, dko, q, k, qw, kw, cosb, sinb, rq, rk, none, none);
}

// As qk_norm_rope_bwd, with the q / k norm weight gradients accumulated into dqw_acc / dkw_acc -> {dq, dk}
std::vector<torch::Tensor> qk_norm_rope_bwd_acc(torch::Tensor dqo, torch::Tensor dko, torch::Tensor q, torch::Tensor k,
                                                torch::Tensor qw, torch::Tensor kw, torch::Tensor cosb,
                                                torch::Tensor sinb, torch::Tensor rq, torch::Tensor rk,
                                                torch::Tensor dqw_acc, torch::Tensor dkw_acc) {
  auto r = qk_norm_rope_bwd_impl(dqo, dko, q, k, qw, kw, cosb, sinb, rq, rk, dqw_acc, dkw_acc);
  return {r[0], r[1]};
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  check_bf16(gu, "gate_up");
  const int F2 = gu.size(-1);
  TORCH_CHECK(F2 % 16 == 0, "swiglu: 2F must be a multiple of 16");
  const int F = F2 / 2;
  const long rows = gu.numel() / F2;
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto y = torch::empty(sizes, gu.options());
  if (rows == 0) return y;
  long total = rows * (F / 8);
  TORCH_CHECK(total < (1l << 31), "swiglu: too many elements");
  int blocks = (int)std::min<long>((total + 255) / 256, (long)sm_count() * 16);
  swiglu_fwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)y.data_ptr(), rows, F);
  BB_POST_LAUNCH();
  return y;
}

torch::Tensor swiglu_bwd(torch::Tensor dy, torch::Tensor gu) {
  check_bf16(dy, "dy");
  check_bf16(gu, "gate_up");
  const int F2 = gu.size(-1), F = F2 / 2;
  const long rows = gu.numel() / F2;
  auto dgu = torch::empty_like(gu);
  if (rows == 0) return dgu;
  long total = rows * (F / 8);
  TORCH_CHECK(total < (1l << 31), "swiglu: too many elements");
  int blocks = (int)std::min<long>((total + 255) / 256, (long)sm_count() * 16);
  swiglu_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)dgu.data_ptr(), rows,
      F);
  BB_POST_LAUNCH();
  return dgu;
}

void logprob_stats(torch::Tensor logits, torch::Tensor targets, torch::Tensor inv_temp, int64_t vocab_start,
                   torch::Tensor stats) {
  check_bf16(logits, "logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && inv_temp.scalar_type() == at::kFloat, "targets/inv_temp dtype");
  const int U = logits.size(0), V = logits.size(1);
  if (U == 0) return;
  TORCH_CHECK(stats.is_contiguous() && stats.size(0) == U && stats.size(1) == 4, "stats must be [U, 4]");
  logprob_stats_kernel<<<U, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)logits.data_ptr(), targets.data_ptr<int64_t>(), inv_temp.data_ptr<float>(),
      stats.data_ptr<float>(), V, (long)vocab_start);
  BB_POST_LAUNCH();
}

std::vector<torch::Tensor> logprob_finalize(torch::Tensor stats) {
  const int U = stats.size(0);
  auto o = stats.options();
  auto lse = torch::empty({U}, o), lp = torch::empty({U}, o), ent = torch::empty({U}, o), ez = torch::empty({U}, o);
  if (U) {
    logprob_finalize_kernel<<<(U + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        stats.data_ptr<float>(), lse.data_ptr<float>(), lp.data_ptr<float>(), ent.data_ptr<float>(),
        ez.data_ptr<float>(), U);
    BB_POST_LAUNCH();
  }
  return {lse, lp, ent, ez};
}

void logprob_grad_inplace(torch::Tensor logits, torch::Tensor targets, torch::Tensor inv_temp, torch::Tensor lse,
                          torch::Tensor ezn, torch::Tensor dlp, c10::optional<torch::Tensor> dent,
                          int64_t vocab_start) {
  check_bf16(logits, "logits");
  const int U = logits.size(0), V = logits.size(1);
  if (U == 0) return;
  const float* dptr = dent.has_value() ? dent->data_ptr<float>() : nullptr;
  logprob_grad_kernel<<<U, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      (__nv_bfloat16*)logits.data_ptr(), targets.data_ptr<int64_t>(), inv_temp.data_ptr<float>(),
      lse.data_ptr<float>(), ezn.data_ptr<float>(), dlp.data_ptr<float>(), dptr, V, (long)vocab_start);
  BB_POST_LAUNCH();
}

std::vector<torch::Tensor> ppo_loss_fwd(torch::Tensor x, torch::Tensor old, torch::Tensor adv,
                                        c10::optional<torch::Tensor> w, double denom, double lo, double hi,
                                        double c) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(), "ppo: x must be fp32 contiguous");
  const long n = x.numel();
  auto out = torch::empty({}, x.options());
  auto grad = torch::empty_like(x);
  auto stats = torch::empty({4}, x.options());
  const int blocks = (int)std::max<long>(1, std::min<long>((n + 1023) / 1024, (long)sm_count() * 2));
  auto part = torch::empty({blocks, 5}, x.options());
  auto stream = at::cuda::getCurrentCUDAStream();
  ppo_loss_kernel<<<blocks, 1024, 0, stream>>>(
      x.data_ptr<float>(), old.data_ptr<float>(), adv.data_ptr<float>(),
      w.has_value() ? w->data_ptr<float>() : nullptr, part.data_ptr<float>(), grad.data_ptr<float>(), n,
      (float)(1.0 / denom), (float)lo, (float)hi, (float)c);
  BB_POST_LAUNCH();
  ppo_loss_finalize_kernel<<<1, 32, 0, stream>>>(part.data_ptr<float>(), blocks, n, (float)(1.0 / denom),
                                                 out.data_ptr<float>(), stats.data_ptr<float>());
  BB_POST_LAUNCH();
  return {out, grad, stats};
}

void adamw_step(torch::Tensor master, torch::Tensor param, torch::Tensor grad, torch::Tensor m, torch::Tensor v,
                torch::Tensor clip, double lr, double b1, double b2, double eps, double wd, double bc1,
                double bc2) {
  const long n = master.numel();
  if (!n) return;
  auto clipf = clip.to(at::kFloat).contiguous();
  auto stream = at::cuda::getCurrentCUDAStream();
  auto al = [](const torch::Tensor& t, uintptr_t a) { return (reinterpret_cast<uintptr_t>(t.data_ptr()) % a) == 0; };
  const bool vec = al(master, 16) && al(grad, 16) && al(m, 16) && al(v, 16) &&
                   al(param, param.scalar_type() == at::kBFloat16 ? 8 : 16);
  const long work = vec ? (n + 3) / 4 : n;
  int blocks = (int)std::min<long>((work + 255) / 256, (long)sm_count() * 8);
  if (param.scalar_type() == at::kBFloat16) {
    adamw_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(
        master.data_ptr<float>(), (__nv_bfloat16*)param.data_ptr(), grad.data_ptr<float>(), m.data_ptr<float>(),
        v.data_ptr<float>(), clipf.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd,
        (float)bc1, (float)bc2, vec);
  } else {
    adamw_kernel<float><<<blocks, 256, 0, stream>>>(
        master.data_ptr<float>(), param.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(),
        v.data_ptr<float>(), clipf.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd,
        (float)bc1, (float)bc2, vec);
  }
  BB_POST_LAUNCH();
}

int64_t bb_launch_count() { return (int64_t)bb::launch_counter().load(); }

// out[0] (+)= sum(x^2) over an FP32 tensor (deterministic; no host sync)
void sumsq_into(torch::Tensor x, torch::Tensor out, bool accumulate) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous(), "sumsq: contiguous CUDA fp32");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.numel() >= 1, "sumsq: fp32 output");
  const long n = x.numel();
  const bool vec = (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) == 0;
  const int blocks = (int)std::max<long>(1, std::min<long>(((vec ? n / 4 : n) + 255) / 256, (long)sm_count() * 8));
  auto part = torch::empty({blocks}, x.options());
  auto stream = at::cuda::getCurrentCUDAStream();
  sumsq_partial_kernel<<<blocks, 256, 0, stream>>>(x.data_ptr<float>(), n, vec, part.data_ptr<float>());
  BB_POST_LAUNCH();
  sum_partials_kernel<<<1, 1024, 0, stream>>>(part.data_ptr<float>(), blocks, out.data_ptr<float>(), accumulate);
  BB_POST_LAUNCH();
}

// out[t] = weight[ids[t] - start] (zero rows for ids outside this rank's [start, start + rows))
torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w, int64_t start) {
  check_bf16(w, "embedding weight");
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.dim() == 1,
              "embedding: ids must be a contiguous CUDA int64 vector");
  const int T = ids.numel(), H = w.size(1);
  TORCH_CHECK(H % 8 == 0, "embedding: hidden size must be a multiple of 8");
  auto out = torch::empty({T, H}, w.options());
  if (T == 0) return out;
  const int blocks = bb::resident_grid(embedding_fwd_kernel, 256, 0, (T + 7) / 8);
  embedding_fwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)out.data_ptr(), T, H, start,
      w.size(0));
  BB_POST_LAUNCH();
  return out;
}

// grad[ids[t] - start] += dy[t] for ids inside this rank's rows; grad is FP32 [rows, H] (e.g. main_grad)
void embedding_bwd_acc(torch::Tensor ids, torch::Tensor dy, torch::Tensor grad, int64_t start) {
  check_bf16(dy, "embedding dy");
  TORCH_CHECK(grad.is_cuda() && grad.scalar_type() == at::kFloat && grad.is_contiguous() && grad.dim() == 2 &&
                  grad.size(1) == dy.size(1) && (reinterpret_cast<uintptr_t>(grad.data_ptr()) & 15) == 0,
              "embedding_bwd: grad must be a contiguous, 16-byte aligned FP32 [rows, H] tensor");
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.is_contiguous() && ids.dim() == 1,
              "embedding_bwd: ids must be a contiguous CUDA int64 vector");
  TORCH_CHECK(dy.dim() == 2 && dy.size(0) == ids.numel() && dy.is_contiguous(),
              "embedding_bwd: dy must be a contiguous [ids.numel(), H] tensor");
  const int T = ids.numel(), H = dy.size(1);
  if (T == 0) return;
  const int blocks = bb::resident_grid(embedding_bwd_acc_kernel, 256, 0, (T + 7) / 8);
  embedding_bwd_acc_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), (const __nv_bfloat16*)dy.data_ptr(), grad.data_ptr<float>(), T, H, start, grad.size(0));
  BB_POST_LAUNCH();
}
