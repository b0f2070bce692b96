// Chunked gated delta rule (Gated DeltaNet), forward and backward, with initial / final state.
//
// Recurrence (per head, FLA convention): S_t = e^{g_t} S_{t-1};  u_t = beta_t (v_t - S_t^T k_t);
// S_t += k_t u_t^T;  o_t = scale * S_t^T q_t.  State S is [K, V] FP32.
//
// The value columns of S evolve independently, so one CTA owns (sequence b, head h, value block of
// VB=32 columns): its state block [K, VB] lives in shared memory for the whole sequence.  Chunks of
// CS=64 tokens use the WY/UT form (G = cumsum g, D_ts = e^{G_t-G_s}):
//   A = D o (K K^T) strictly lower,  T = (I + diag(beta) A)^-1,
//   Wk = T diag(beta e^G) K,  U = T diag(beta) V - Wk S0,
//   O = scale (diag(e^G) Q S0 + (D o Q K^T)_{s<=t} U),   S1 = e^{G_n} S0 + K^T diag(e^{G_n-G}) U.
// Forward checkpoints S0 of every chunk (FP32) for the backward, which walks the chunks in reverse,
// recomputes the chunk intermediates and applies the hand-derived adjoint of every line above.
// dq / dk / dg / dbeta are sums over value blocks (FP32 atomics); dv and dh0 are written by their owner.
//
// Matrix products run on CUDA cores from padded shared memory (FP32 accumulation); q/k are kept as
// bf16 in shared memory (exact copies of the inputs).
//
// Parity: MindSpeed-Ops chunk_gated_delta_rule (chunk 64, head_first=False, initial_state /
// output_final_state, dh0 / dht) as called from verl/models/mcore/tpr/gated_delta_net.py:239-263.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace {

constexpr int CS = 64;
constexpr int VB = 32;
constexpr int NT = 256;

template <int K>
struct Lay {
  static constexpr int LQ = K + 2;   // bf16 row stride (odd word count -> conflict-free column walks)
  static constexpr int LW = K + 1;   // fp32 [CS][K]
  static constexpr int LS = VB + 1;  // fp32 [K][VB] and [CS][VB]
  static constexpr int LN = CS + 1;  // fp32 [CS][CS]
};

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

template <int K>
__device__ __forceinline__ float dotqk(const __nv_bfloat16* a, const __nv_bfloat16* b) {
  float s = 0.f;
#pragma unroll 8
  for (int i = 0; i < K; ++i) s += bf(a[i]) * bf(b[i]);
  return s;
}

// Load one chunk of q, k (bf16 rows), v block, g, beta; rows >= n are zero.
template <int K>
__device__ void load_chunk(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                           const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
                           const float* __restrict__ beta, int row0, int n, int H, int V, int h, int v0,
                           __nv_bfloat16* sQ, __nv_bfloat16* sK, float* sV, float* sG, float* sB) {
  using LY = Lay<K>;
  for (int i = threadIdx.x; i < CS * K; i += NT) {
    const int t = i / K, c = i % K;
    const bool ok = t < n;
    const size_t off = ((size_t)(row0 + t) * H + h) * K + c;
    sQ[t * LY::LQ + c] = ok ? q[off] : __float2bfloat16(0.f);
    sK[t * LY::LQ + c] = ok ? k[off] : __float2bfloat16(0.f);
  }
  for (int i = threadIdx.x; i < CS * VB; i += NT) {
    const int t = i / VB, j = i % VB;
    sV[t * LY::LS + j] = t < n ? bf(v[((size_t)(row0 + t) * H + h) * V + v0 + j]) : 0.f;
  }
  for (int t = threadIdx.x; t < CS; t += NT) {
    sG[t] = t < n ? g[(size_t)(row0 + t) * H + h] : 0.f;
    sB[t] = t < n ? beta[(size_t)(row0 + t) * H + h] : 0.f;
  }
}

// G = cumsum(g) (in place), Gam = exp(G), E = exp(G_last - G).
__device__ void chunk_scan(float* sG, float* sGam, float* sE, int n) {
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int t = 0; t < CS; ++t) {
      acc += sG[t];
      sG[t] = acc;
    }
  }
  __syncthreads();
  const float gl = sG[max(n - 1, 0)];
  for (int t = threadIdx.x; t < CS; t += NT) {
    sGam[t] = t < n ? __expf(sG[t]) : 0.f;
    sE[t] = t < n ? __expf(gl - sG[t]) : 0.f;
  }
  __syncthreads();
}

// A (strictly lower, D o KK^T) and T = (I + diag(beta) A)^-1 (lower, unit diagonal).
template <int K>
__device__ void build_A_T(const __nv_bfloat16* sK, const float* sG, const float* sB, float* sA, float* sT, int n) {
  using LY = Lay<K>;
  for (int i = threadIdx.x; i < CS * CS; i += NT) {
    const int t = i / CS, s = i % CS;
    float a = 0.f;
    if (s < t && t < n) a = __expf(sG[t] - sG[s]) * dotqk<K>(sK + t * LY::LQ, sK + s * LY::LQ);
    sA[t * LY::LN + s] = a;
    sT[t * LY::LN + s] = 0.f;
  }
  __syncthreads();
  // forward substitution, row by row: T[t, j] = [t==j] - beta_t sum_{j<=s<t} A[t, s] T[s, j]
  for (int t = 0; t < n; ++t) {
    for (int j = threadIdx.x; j <= t; j += NT) {
      float acc = 0.f;
      for (int s = j; s < t; ++s) acc += sA[t * LY::LN + s] * sT[s * LY::LN + j];
      sT[t * LY::LN + j] = (t == j ? 1.f : 0.f) - sB[t] * acc;
    }
    __syncthreads();
  }
}

// Wk = T diag(beta Gam) K  [CS x K];  U = T diag(beta) V - Wk S0  [CS x VB]
template <int K>
__device__ void build_W_U(const __nv_bfloat16* sK, const float* sT, const float* sB, const float* sGam,
                          const float* sV, const float* sS, float* sW, float* sU, int n) {
  using LY = Lay<K>;
  for (int i = threadIdx.x; i < CS * K; i += NT) {
    const int t = i / K, c = i % K;
    float acc = 0.f;
    if (t < n)
      for (int s = 0; s <= t; ++s) acc += sT[t * LY::LN + s] * sB[s] * sGam[s] * bf(sK[s * LY::LQ + c]);
    sW[t * LY::LW + c] = acc;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < CS * VB; i += NT) {
    const int t = i / VB, j = i % VB;
    float acc = 0.f;
    if (t < n) {
      for (int s = 0; s <= t; ++s) acc += sT[t * LY::LN + s] * sB[s] * sV[s * LY::LS + j];
      for (int c = 0; c < K; ++c) acc -= sW[t * LY::LW + c] * sS[c * LY::LS + j];
    }
    sU[t * LY::LS + j] = acc;
  }
  __syncthreads();
}

template <int K>
struct FwdSmem {
  using LY = Lay<K>;
  static constexpr size_t Q = 0;
  static constexpr size_t KK = Q + sizeof(__nv_bfloat16) * CS * LY::LQ;
  static constexpr size_t W = KK + sizeof(__nv_bfloat16) * CS * LY::LQ;
  static constexpr size_t S = W + sizeof(float) * CS * LY::LW;
  static constexpr size_t V = S + sizeof(float) * K * LY::LS;
  static constexpr size_t U = V + sizeof(float) * CS * LY::LS;
  static constexpr size_t A = U + sizeof(float) * CS * LY::LS;
  static constexpr size_t T = A + sizeof(float) * CS * LY::LN;
  static constexpr size_t VEC = T + sizeof(float) * CS * LY::LN;  // G, B, Gam, E
  static constexpr size_t TOTAL = VEC + sizeof(float) * 4 * CS;
};

template <int K>
__global__ void __launch_bounds__(NT) gdr_fwd_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, const float* __restrict__ h0,
    const int* __restrict__ cu, __nv_bfloat16* __restrict__ o, float* __restrict__ hT, float* __restrict__ ckpt,
    int H, int V, int nc_max, float scale) {
  using LY = Lay<K>;
  using SM = FwdSmem<K>;
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem + SM::Q);
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem + SM::KK);
  float* sW = reinterpret_cast<float*>(smem + SM::W);
  float* sS = reinterpret_cast<float*>(smem + SM::S);
  float* sV = reinterpret_cast<float*>(smem + SM::V);
  float* sU = reinterpret_cast<float*>(smem + SM::U);
  float* sA = reinterpret_cast<float*>(smem + SM::A);
  float* sT = reinterpret_cast<float*>(smem + SM::T);
  float* sG = reinterpret_cast<float*>(smem + SM::VEC);
  float* sB = sG + CS;
  float* sGam = sB + CS;
  float* sE = sGam + CS;

  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vb * VB;
  const int q0 = cu[b], L = cu[b + 1] - q0;
  const int nch = (L + CS - 1) / CS;
  for (int i = threadIdx.x; i < K * VB; i += NT) {
    const int c = i / VB, j = i % VB;
    sS[c * LY::LS + j] = h0 ? h0[(((size_t)b * H + h) * K + c) * V + v0 + j] : 0.f;
  }
  __syncthreads();
  for (int ch = 0; ch < nch; ++ch) {
    const int t0 = ch * CS, n = min(CS, L - t0);
    float* ck = ckpt + ((((size_t)b * H + h) * nc_max + ch) * K) * V;
    for (int i = threadIdx.x; i < K * VB; i += NT) {
      const int c = i / VB, j = i % VB;
      ck[(size_t)c * V + v0 + j] = sS[c * LY::LS + j];
    }
    load_chunk<K>(q, k, v, g, beta, q0 + t0, n, H, V, h, v0, sQ, sK, sV, sG, sB);
    __syncthreads();
    chunk_scan(sG, sGam, sE, n);
    build_A_T<K>(sK, sG, sB, sA, sT, n);
    build_W_U<K>(sK, sT, sB, sGam, sV, sS, sW, sU, n);
    // P = D o (Q K^T) for s <= t (into sA; A is no longer needed)
    for (int i = threadIdx.x; i < CS * CS; i += NT) {
      const int t = i / CS, s = i % CS;
      float p = 0.f;
      if (s <= t && t < n) p = __expf(sG[t] - sG[s]) * dotqk<K>(sQ + t * LY::LQ, sK + s * LY::LQ);
      sA[t * LY::LN + s] = p;
    }
    __syncthreads();
    // O = scale (Gam o (Q S0) + P U)
    for (int i = threadIdx.x; i < CS * VB; i += NT) {
      const int t = i / VB, j = i % VB;
      if (t >= n) continue;
      float qs = 0.f;
      for (int c = 0; c < K; ++c) qs += bf(sQ[t * LY::LQ + c]) * sS[c * LY::LS + j];
      float pu = 0.f;
      for (int s = 0; s <= t; ++s) pu += sA[t * LY::LN + s] * sU[s * LY::LS + j];
      o[((size_t)(q0 + t0 + t) * H + h) * V + v0 + j] = __float2bfloat16(scale * (sGam[t] * qs + pu));
    }
    __syncthreads();
    // S1 = Gam_last S0 + K^T diag(E) U
    const float gl = sGam[n - 1];
    for (int i = threadIdx.x; i < K * VB; i += NT) {
      const int c = i / VB, j = i % VB;
      float acc = gl * sS[c * LY::LS + j];
      for (int t = 0; t < n; ++t) acc += bf(sK[t * LY::LQ + c]) * sE[t] * sU[t * LY::LS + j];
      sS[c * LY::LS + j] = acc;
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < K * VB; i += NT) {
    const int c = i / VB, j = i % VB;
    hT[(((size_t)b * H + h) * K + c) * V + v0 + j] = sS[c * LY::LS + j];
  }
}

template <int K>
struct BwdSmem {
  using LY = Lay<K>;
  static constexpr size_t Q = 0;
  static constexpr size_t KK = Q + sizeof(__nv_bfloat16) * CS * LY::LQ;
  static constexpr size_t W = KK + sizeof(__nv_bfloat16) * CS * LY::LQ;  // Wk, then dWk, then dKb
  static constexpr size_t S0 = W + sizeof(float) * CS * LY::LW;
  static constexpr size_t DS = S0 + sizeof(float) * K * LY::LS;
  static constexpr size_t V = DS + sizeof(float) * K * LY::LS;
  static constexpr size_t DO = V + sizeof(float) * CS * LY::LS;
  static constexpr size_t U = DO + sizeof(float) * CS * LY::LS;
  static constexpr size_t DU = U + sizeof(float) * CS * LY::LS;
  static constexpr size_t A = DU + sizeof(float) * CS * LY::LS;
  static constexpr size_t T = A + sizeof(float) * CS * LY::LN;
  static constexpr size_t P = T + sizeof(float) * CS * LY::LN;
  static constexpr size_t DP = P + sizeof(float) * CS * LY::LN;
  static constexpr size_t VEC = DP + sizeof(float) * CS * LY::LN;  // G B Gam E dG dB dGam de
  static constexpr size_t TOTAL = VEC + sizeof(float) * 8 * CS + 16;
};

template <int K>
__global__ void __launch_bounds__(NT) gdr_bwd_kernel(
    const __nv_bfloat16* __restrict__ dout, const float* __restrict__ dhT, const __nv_bfloat16* __restrict__ q,
    const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, const float* __restrict__ ckpt, const int* __restrict__ cu,
    float* __restrict__ dq, float* __restrict__ dk, __nv_bfloat16* __restrict__ dv, float* __restrict__ dg,
    float* __restrict__ dbeta, float* __restrict__ dh0, int H, int V, int nc_max, float scale) {
  using LY = Lay<K>;
  using SM = BwdSmem<K>;
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem + SM::Q);
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem + SM::KK);
  float* sW = reinterpret_cast<float*>(smem + SM::W);
  float* sS0 = reinterpret_cast<float*>(smem + SM::S0);
  float* sdS = reinterpret_cast<float*>(smem + SM::DS);
  float* sV = reinterpret_cast<float*>(smem + SM::V);
  float* sdO = reinterpret_cast<float*>(smem + SM::DO);
  float* sU = reinterpret_cast<float*>(smem + SM::U);
  float* sdU = reinterpret_cast<float*>(smem + SM::DU);
  float* sA = reinterpret_cast<float*>(smem + SM::A);
  float* sT = reinterpret_cast<float*>(smem + SM::T);
  float* sP = reinterpret_cast<float*>(smem + SM::P);
  float* sdP = reinterpret_cast<float*>(smem + SM::DP);
  float* sG = reinterpret_cast<float*>(smem + SM::VEC);
  float* sB = sG + CS;
  float* sGam = sB + CS;
  float* sE = sGam + CS;
  float* sdG = sE + CS;
  float* sdB = sdG + CS;
  float* sdGam = sdB + CS;
  float* sde = sdGam + CS;
  float* sRed = sde + CS;  // 1 float: <dS1, S0>

  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vb * VB;
  const int q0 = cu[b], L = cu[b + 1] - q0;
  const int nch = (L + CS - 1) / CS;
  for (int i = threadIdx.x; i < K * VB; i += NT) {
    const int c = i / VB, j = i % VB;
    sdS[c * LY::LS + j] = dhT ? dhT[(((size_t)b * H + h) * K + c) * V + v0 + j] : 0.f;
  }
  __syncthreads();
  for (int ch = nch - 1; ch >= 0; --ch) {
    const int t0 = ch * CS, n = min(CS, L - t0);
    const float* ck = ckpt + ((((size_t)b * H + h) * nc_max + ch) * K) * V;
    for (int i = threadIdx.x; i < K * VB; i += NT) {
      const int c = i / VB, j = i % VB;
      sS0[c * LY::LS + j] = ck[(size_t)c * V + v0 + j];
    }
    load_chunk<K>(q, k, v, g, beta, q0 + t0, n, H, V, h, v0, sQ, sK, sV, sG, sB);
    for (int i = threadIdx.x; i < CS * VB; i += NT) {
      const int t = i / VB, j = i % VB;
      sdO[t * LY::LS + j] = t < n ? bf(dout[((size_t)(q0 + t0 + t) * H + h) * V + v0 + j]) : 0.f;
    }
    for (int t = threadIdx.x; t < CS; t += NT) sdG[t] = sdB[t] = sdGam[t] = sde[t] = 0.f;
    if (threadIdx.x == 0) sRed[0] = 0.f;
    __syncthreads();
    chunk_scan(sG, sGam, sE, n);
    build_A_T<K>(sK, sG, sB, sA, sT, n);
    build_W_U<K>(sK, sT, sB, sGam, sV, sS0, sW, sU, n);
    // P = D o QK^T (s <= t)
    for (int i = threadIdx.x; i < CS * CS; i += NT) {
      const int t = i / CS, s = i % CS;
      float p = 0.f;
      if (s <= t && t < n) p = __expf(sG[t] - sG[s]) * dotqk<K>(sQ + t * LY::LQ, sK + s * LY::LQ);
      sP[t * LY::LN + s] = p;
    }
    __syncthreads();
    // dU = scale P^T dO + E o (K dS);  de_s = sum_j (K dS)[s,j] U[s,j]
    for (int i = threadIdx.x; i < CS * VB; i += NT) {
      const int s = i / VB, j = i % VB;
      float a = 0.f, kds = 0.f;
      if (s < n) {
        for (int t = s; t < n; ++t) a += sP[t * LY::LN + s] * sdO[t * LY::LS + j];
        for (int c = 0; c < K; ++c) kds += bf(sK[s * LY::LQ + c]) * sdS[c * LY::LS + j];
      }
      sdU[s * LY::LS + j] = scale * a + sE[s] * kds;
      if (s < n) atomicAdd(&sde[s], kds * sU[s * LY::LS + j]);
    }
    // dP = scale dO U^T (s <= t);  <dS1, S0>
    for (int i = threadIdx.x; i < CS * CS; i += NT) {
      const int t = i / CS, s = i % CS;
      float a = 0.f;
      if (s <= t && t < n)
        for (int j = 0; j < VB; ++j) a += sdO[t * LY::LS + j] * sU[s * LY::LS + j];
      sdP[t * LY::LN + s] = scale * a;
    }
    {
      float part = 0.f;
      for (int i = threadIdx.x; i < K * VB; i += NT) {
        const int c = i / VB, j = i % VB;
        part += sdS[c * LY::LS + j] * sS0[c * LY::LS + j];
      }
      part = bb::warp_sum(part);
      if ((threadIdx.x & 31) == 0) atomicAdd(sRed, part);
    }
    __syncthreads();
    // dGam_t += scale <(Q S0)_t, dO_t>;  dG from P: (dD o D)_ts = dP_ts P_ts
    for (int t = threadIdx.x; t < n; t += NT) {
      float a = 0.f;
      for (int j = 0; j < VB; ++j) {
        float qs = 0.f;
        for (int c = 0; c < K; ++c) qs += bf(sQ[t * LY::LQ + c]) * sS0[c * LY::LS + j];
        a += qs * sdO[t * LY::LS + j];
      }
      float rs = 0.f, cs = 0.f;
      for (int s = 0; s <= t; ++s) rs += sdP[t * LY::LN + s] * sP[t * LY::LN + s];
      for (int u = t; u < n; ++u) cs += sdP[u * LY::LN + t] * sP[u * LY::LN + t];
      sdGam[t] += scale * a;
      sdG[t] += rs - cs;
    }
    // dQ (this value block's share): scale Gam_t dO_t S0^T + (dP o D) K ;  dK from P: (dP o D)^T Q
    for (int i = threadIdx.x; i < CS * K; i += NT) {
      const int t = i / K, c = i % K;
      if (t >= n) continue;
      float a = 0.f;
      for (int j = 0; j < VB; ++j) a += sdO[t * LY::LS + j] * sS0[c * LY::LS + j];
      a *= scale * sGam[t];
      float bq = 0.f, bk = 0.f;
      for (int s = 0; s <= t; ++s) bq += sdP[t * LY::LN + s] * __expf(sG[t] - sG[s]) * bf(sK[s * LY::LQ + c]);
      for (int u = t; u < n; ++u) bk += sdP[u * LY::LN + t] * __expf(sG[u] - sG[t]) * bf(sQ[u * LY::LQ + c]);
      // dK from S1 = ... K^T E U:  E_t (U_t . dS_c)
      float ks = 0.f;
      for (int j = 0; j < VB; ++j) ks += sU[t * LY::LS + j] * sdS[c * LY::LS + j];
      const size_t off = ((size_t)(q0 + t0 + t) * H + h) * K + c;
      atomicAdd(&dq[off], a + bq);
      atomicAdd(&dk[off], bk + sE[t] * ks);
    }
    __syncthreads();
    // dS0 = scale Q^T (Gam o dO) + Gam_last dS - Wk^T dU   (written into sdS after all uses of dS1)
    const float gl = sGam[n - 1];
    // dGam_last += <dS1, S0>; de-terms: dG_last += sum de E, dG_t -= de_t E_t
    if (threadIdx.x == 0) {
      float tot = 0.f;
      for (int t = 0; t < n; ++t) tot += sde[t] * sE[t];
      sdGam[n - 1] += sRed[0];
      sdG[n - 1] += tot;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < n; t += NT) sdG[t] -= sde[t] * sE[t];
    for (int i = threadIdx.x; i < K * VB; i += NT) {
      const int c = i / VB, j = i % VB;
      float a = 0.f, w = 0.f;
      for (int t = 0; t < n; ++t) {
        a += bf(sQ[t * LY::LQ + c]) * sGam[t] * sdO[t * LY::LS + j];
        w += sW[t * LY::LW + c] * sdU[t * LY::LS + j];
      }
      sdS[c * LY::LS + j] = scale * a + gl * sdS[c * LY::LS + j] - w;
    }
    __syncthreads();
    // dT = dU (beta o V)^T + dWk (beta Gam o K)^T with dWk = -dU S0^T  (into sA's twin: reuse sP)
    for (int i = threadIdx.x; i < CS * K; i += NT) {
      const int t = i / K, c = i % K;
      float a = 0.f;
      if (t < n)
        for (int j = 0; j < VB; ++j) a += sdU[t * LY::LS + j] * sS0[c * LY::LS + j];
      sW[t * LY::LW + c] = -a;  // dWk
    }
    __syncthreads();
    for (int i = threadIdx.x; i < CS * CS; i += NT) {
      const int t = i / CS, s = i % CS;
      float a = 0.f;
      if (t < n && s < n) {
        for (int j = 0; j < VB; ++j) a += sdU[t * LY::LS + j] * sB[s] * sV[s * LY::LS + j];
        for (int c = 0; c < K; ++c) a += sW[t * LY::LW + c] * sB[s] * sGam[s] * bf(sK[s * LY::LQ + c]);
      }
      sP[t * LY::LN + s] = a;  // dT
    }
    __syncthreads();
    // dVb = T^T dU -> dv = beta o dVb, dbeta += <v, dVb>;  dKb = T^T dWk (into sU's role: compute per element)
    for (int i = threadIdx.x; i < CS * VB; i += NT) {
      const int s = i / VB, j = i % VB;
      if (s >= n) continue;
      float a = 0.f;
      for (int t = s; t < n; ++t) a += sT[t * LY::LN + s] * sdU[t * LY::LS + j];
      dv[((size_t)(q0 + t0 + s) * H + h) * V + v0 + j] = __float2bfloat16(sB[s] * a);
      atomicAdd(&sdB[s], a * sV[s * LY::LS + j]);
    }
    for (int i = threadIdx.x; i < CS * K; i += NT) {
      const int s = i / K, c = i % K;
      if (s >= n) continue;
      float a = 0.f;
      for (int t = s; t < n; ++t) a += sT[t * LY::LN + s] * sW[t * LY::LW + c];
      const float kv = bf(sK[s * LY::LQ + c]);
      atomicAdd(&dk[((size_t)(q0 + t0 + s) * H + h) * K + c], sB[s] * sGam[s] * a);
      const float r = kv * a;
      atomicAdd(&sdB[s], sGam[s] * r);
      atomicAdd(&sdGam[s], sB[s] * r);
    }
    __syncthreads();
    // dL = -T^T dT T^T  (two triangular products; dT lives in sP, result into sdP)
    for (int i = threadIdx.x; i < CS * CS; i += NT) {  // X = dT T^T  (into sdP temporarily)
      const int t = i / CS, s = i % CS;
      float a = 0.f;
      if (t < n && s < n)
        for (int u = 0; u <= s; ++u) a += sP[t * LY::LN + u] * sT[s * LY::LN + u];
      sdP[t * LY::LN + s] = a;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < CS * CS; i += NT) {  // dL = -T^T X  (into sP)
      const int t = i / CS, s = i % CS;
      float a = 0.f;
      if (t < n && s < n)
        for (int u = t; u < n; ++u) a += sT[u * LY::LN + t] * sdP[u * LY::LN + s];
      sP[t * LY::LN + s] = -a;
    }
    __syncthreads();
    // dA_ts = beta_t dL_ts (s < t); dbeta_t += sum_s dL_ts A_ts; dG from A: (dA o A);  dKK = dA o D
    for (int t = threadIdx.x; t < n; t += NT) {
      float r = 0.f, rs = 0.f;
      for (int s = 0; s < t; ++s) {
        r += sP[t * LY::LN + s] * sA[t * LY::LN + s];
        rs += sB[t] * sP[t * LY::LN + s] * sA[t * LY::LN + s];
      }
      float cs = 0.f;
      for (int u = t + 1; u < n; ++u) cs += sB[u] * sP[u * LY::LN + t] * sA[u * LY::LN + t];
      sdB[t] += r;
      sdG[t] += rs - cs;
    }
    for (int i = threadIdx.x; i < CS * K; i += NT) {
      const int t = i / K, c = i % K;
      if (t >= n) continue;
      float a = 0.f;
      for (int s = 0; s < n; ++s) {
        if (s == t) continue;
        const int hi = max(t, s), lo = min(t, s);
        const float dkk = sB[hi] * sP[hi * LY::LN + lo] * __expf(sG[hi] - sG[lo]);
        a += dkk * bf(sK[s * LY::LQ + c]);
      }
      atomicAdd(&dk[((size_t)(q0 + t0 + t) * H + h) * K + c], a);
    }
    __syncthreads();
    // dG_t += dGam_t Gam_t; dg = reverse cumsum(dG); flush dbeta
    if (threadIdx.x == 0) {
      float acc = 0.f;
      for (int t = n - 1; t >= 0; --t) {
        acc += sdG[t] + sdGam[t] * sGam[t];
        atomicAdd(&dg[(size_t)(q0 + t0 + t) * H + h], acc);
        atomicAdd(&dbeta[(size_t)(q0 + t0 + t) * H + h], sdB[t]);
      }
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < K * VB; i += NT) {
    const int c = i / VB, j = i % VB;
    if (dh0) dh0[(((size_t)b * H + h) * K + c) * V + v0 + j] = sdS[c * LY::LS + j];
  }
}

template <int K>
void set_smem(const void* kern, size_t bytes) {
  BB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

}  // namespace

std::vector<torch::Tensor> gdr_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                   torch::Tensor beta, c10::optional<torch::Tensor> h0, torch::Tensor cu,
                                   int64_t max_len, double scale, int64_t chunk) {
  TORCH_CHECK(chunk == CS, "gated delta rule kernel uses chunk 64");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
              "gdr: q/k/v contiguous bf16");
  const int T = q.size(0), H = q.size(1), K = q.size(2), V = v.size(2);
  TORCH_CHECK(V % VB == 0, "gdr: value dim must be a multiple of 32");
  const int B = cu.numel() - 1;
  const int nc = (int)((max_len + CS - 1) / CS);
  auto o = torch::empty_like(v);
  auto hT = torch::empty({B, H, K, V}, q.options().dtype(at::kFloat));
  auto ckpt = torch::empty({B, H, std::max(nc, 1), K, V}, q.options().dtype(at::kFloat));
  if (T == 0 || B == 0) return {o, hT, ckpt};
  auto gf = g.to(at::kFloat).contiguous(), bf_ = beta.to(at::kFloat).contiguous();
  torch::Tensor h0f;
  if (h0.has_value()) h0f = h0->to(at::kFloat).contiguous();
  dim3 grid(V / VB, H, B);
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_GF(KK)                                                                                            \
  {                                                                                                          \
    auto kern = gdr_fwd_kernel<KK>;                                                                          \
    set_smem<KK>((const void*)kern, FwdSmem<KK>::TOTAL);                                                     \
    kern<<<grid, NT, FwdSmem<KK>::TOTAL, stream>>>(                                                          \
        (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(), \
        gf.data_ptr<float>(), bf_.data_ptr<float>(), h0.has_value() ? h0f.data_ptr<float>() : nullptr,          \
        cu.data_ptr<int>(), (__nv_bfloat16*)o.data_ptr(), hT.data_ptr<float>(), ckpt.data_ptr<float>(), H, V,  \
        std::max(nc, 1), (float)scale);                                                                      \
  }
  if (K == 128) BB_GF(128)
  else if (K == 64) BB_GF(64)
  else if (K == 32) BB_GF(32)
  else TORCH_CHECK(false, "gdr: key dim must be 32, 64 or 128");
#undef BB_GF
  BB_POST_LAUNCH();
  return {o, hT, ckpt};
}

std::vector<torch::Tensor> gdr_bwd(torch::Tensor dout, c10::optional<torch::Tensor> dhT, torch::Tensor q,
                                   torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                                   torch::Tensor ckpt, torch::Tensor cu, int64_t max_len, bool has_h0, double scale) {
  const int T = q.size(0), H = q.size(1), K = q.size(2), V = v.size(2);
  const int B = cu.numel() - 1;
  const int nc = (int)((max_len + CS - 1) / CS);
  auto dq = torch::zeros({T, H, K}, q.options().dtype(at::kFloat));
  auto dk = torch::zeros({T, H, K}, q.options().dtype(at::kFloat));
  auto dv = torch::empty_like(v);
  auto dg = torch::zeros({T, H}, q.options().dtype(at::kFloat));
  auto db = torch::zeros({T, H}, q.options().dtype(at::kFloat));
  auto dh0 = torch::zeros({B, H, K, V}, q.options().dtype(at::kFloat));
  if (T == 0 || B == 0) return {dq, dk, dv, dg, db, dh0};
  auto gf = g.to(at::kFloat).contiguous(), bf_ = beta.to(at::kFloat).contiguous();
  auto doc = dout.contiguous();
  torch::Tensor dhTf;
  if (dhT.has_value()) dhTf = dhT->to(at::kFloat).contiguous();
  dim3 grid(V / VB, H, B);
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_GB(KK)                                                                                              \
  {                                                                                                            \
    auto kern = gdr_bwd_kernel<KK>;                                                                            \
    set_smem<KK>((const void*)kern, BwdSmem<KK>::TOTAL);                                                       \
    kern<<<grid, NT, BwdSmem<KK>::TOTAL, stream>>>(                                                            \
        (const __nv_bfloat16*)doc.data_ptr(), dhT.has_value() ? dhTf.data_ptr<float>() : nullptr,              \
        (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(), \
        gf.data_ptr<float>(), bf_.data_ptr<float>(), ckpt.data_ptr<float>(), cu.data_ptr<int>(),                 \
        dq.data_ptr<float>(), dk.data_ptr<float>(), (__nv_bfloat16*)dv.data_ptr(), dg.data_ptr<float>(),         \
        db.data_ptr<float>(), has_h0 ? dh0.data_ptr<float>() : nullptr, H, V, std::max(nc, 1), (float)scale);    \
  }
  if (K == 128) BB_GB(128)
  else if (K == 64) BB_GB(64)
  else if (K == 32) BB_GB(32)
  else TORCH_CHECK(false, "gdr: key dim must be 32, 64 or 128");
#undef BB_GB
  BB_POST_LAUNCH();
  return {dq, dk, dv, dg, db, dh0};
}
