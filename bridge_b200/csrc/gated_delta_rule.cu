// Chunked gated delta rule (Gated DeltaNet) on bf16 tensor cores, forward and backward, varlen,
// with initial / final state.
//
// Recurrence (per head, FLA convention): S_t = e^{g_t} S_{t-1};  u_t = beta_t (v_t - S_t^T k_t);
// S_t += k_t u_t^T;  o_t = scale * S_t^T q_t.  State S is [K, V] FP32.
//
// Chunks of C = 64 tokens (G = cumsum g inside the chunk, Gam = e^G, D_ts = e^{G_t - G_s},
// E_t = e^{G_last - G_t}):
//   A = D o (K K^T) strictly lower,  T = (I + diag(beta) A)^-1,
//   Wk = T diag(beta Gam) K,  Wv = T diag(beta) V,  U = Wv - Wk S0,
//   O = scale (diag(Gam) Q S0 + (D o Q K^T)_{s<=t} U),   S1 = Gam_last S0 + K^T diag(E) U.
// Everything except the S0 -> S1 chain is independent per chunk, so the work is split into
//   gdr_prep_kernel       per (chunk, head):          A, T (blocked 16x16 inverse), Wk, Wv
//   gdr_scan_kernel       per (sequence, head, V blk): the state chain; U, O, S1; FP32 chunk states
//   gdr_bwd_scan_kernel   per (sequence, head, V blk): reverse chain of dS; dU, dWk and the
//                                                      state-dependent parts of dq / dk / dG
//   gdr_bwd_chunk_kernel  per (chunk, head):          everything else (through dP, dT, dL = -T^T dT T^T)
// and every matrix product runs on mma.sync bf16 tensor cores with FP32 accumulation; the chained
// FP32 states (S0, dS1) enter the tensor cores as bf16 hi + lo pairs (two passes) so the chain keeps
// ~16 significant bits instead of bf16's 8.  Gradients
// shared by the V blocks of one head (dq, dk, dWk, dG) are summed with FP32 atomics in the scan
// kernels and finished by the chunk kernel, which owns its rows.
//
// Parity: MindSpeed-Ops chunk_gated_delta_rule (chunk 64, head_first=False, initial_state /
// output_final_state, dh0 / dht) as called from verl/models/mcore/tpr/gated_delta_net.py:239-263.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "warp_mma.cuh"

namespace {

constexpr int CS = 64;
constexpr int NT = 256;
using bf = __nv_bfloat16;

__device__ __forceinline__ float b2f(bf x) { return __bfloat162float(x); }
__device__ __forceinline__ bf f2b(float x) { return __float2bfloat16(x); }

// four consecutive bf16 (8-byte aligned) <-> float4
__device__ __forceinline__ float4 ld_bf4(const bf* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st_bf4(bf* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ float4 scale4(float4 v, float s) { return make_float4(s * v.x, s * v.y, s * v.z, s * v.w); }
// the bf16 rounding of each element, back in FP32
__device__ __forceinline__ float4 ld_bf4_round(float4 v) {
  return make_float4(b2f(f2b(v.x)), b2f(f2b(v.y)), b2f(f2b(v.z)), b2f(f2b(v.w)));
}

// Optional phase timing, off unless enabled from the host (gdr_phase_profile): after a block barrier,
// thread 0 adds the SM cycles the block spent in each phase to a device table [kernel][phase].
// Kernels: 0 prep, 1 scan, 2 bwd scan, 3 bwd chunk.
__device__ int g_gdr_prof_on;
__device__ unsigned long long g_gdr_prof[4][16];

struct PhaseClock {
  bool on = false;
  long long t = 0;
  __device__ __forceinline__ PhaseClock() {
#if defined(__CUDA_ARCH__)
    on = g_gdr_prof_on != 0;
    if (on) t = clock64();
#endif
  }
  __device__ __forceinline__ void mark(int kern, int phase) {
#if defined(__CUDA_ARCH__)
    if (!on) return;
    __syncthreads();
    if (threadIdx.x == 0) {
      const long long now = clock64();
      atomicAdd(&g_gdr_prof[kern][phase], (unsigned long long)(now - t));
      t = now;
    }
#endif
  }
};

struct Chunk {
  int row0, n, b, c;
};

__device__ __forceinline__ Chunk load_chunk_desc(const int* chunks, int i) {
  const int4 d = reinterpret_cast<const int4*>(chunks)[i];
  return {d.x, d.y, d.z, d.w};
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  const int bytes = valid ? 16 : 0;   // 0: nothing is read, the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// rows [row0, row0+n) of a [T, H, W] bf16 tensor (head h, columns [c0, c0+w)) -> smem [64][ld]; zero rows >= n.
// Asynchronous (cp.async): every load of a phase is in flight at once; chunk_decay, which every kernel
// runs before reading the rows, waits for them.
template <int W>
__device__ __forceinline__ void load_rows(bf* dst, int ld, const bf* __restrict__ src, int row0, int n, int H, int h,
                                          int width, int c0) {
  constexpr int VEC = W / 8;
#pragma unroll 4
  for (int i = threadIdx.x; i < CS * VEC; i += NT) {
    const int t = i / VEC, v = i % VEC;
    const bf* g = src + ((size_t)(row0 + (t < n ? t : 0)) * H + h) * width + c0 + v * 8;
    cp_async16(dst + t * ld + v * 8, g, t < n);
  }
}

// G = cumsum(g) over the chunk (rows >= n hold the last value), Gam = e^G, E = e^{G_last - G}.
template <bool WAIT_LOADS = true>
__device__ __forceinline__ void chunk_decay(const float* __restrict__ g, int row0, int n, int H, int h, float* sG,
                                            float* sGam, float* sE) {
  if (WAIT_LOADS) cp_async_wait_all();  // this thread's load_rows copies (made visible by the barriers below)
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float a = lane < n ? g[(size_t)(row0 + lane) * H + h] : 0.f;
    float b = lane + 32 < n ? g[(size_t)(row0 + lane + 32) * H + h] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float ya = __shfl_up_sync(0xffffffffu, a, o), yb = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) {
        a += ya;
        b += yb;
      }
    }
    b += __shfl_sync(0xffffffffu, a, 31);
    sG[lane] = a;
    sG[lane + 32] = b;
  }
  __syncthreads();
  const float gl = sG[max(n - 1, 0)];
  for (int t = threadIdx.x; t < CS; t += NT) {
    sGam[t] = t < n ? __expf(sG[t]) : 0.f;
    sE[t] = t < n ? __expf(gl - sG[t]) : 0.f;
  }
  __syncthreads();
}

// sA (fp32 [64][65]) = D o K K^T strictly lower (raw, without beta); sTf = (I + diag(beta) A)^-1 (fp32);
// sTb = bf16(sTf) with rows >= n zeroed.  The inverse is blocked by 16: each of the first four warps
// inverts one unit-lower diagonal block by warp-synchronous substitution, then the off-diagonal
// blocks follow level by level, T_ij = -T_ii sum_{j<=k<i} L_ik T_kj (L_ik = diag(beta) A block).
template <int KD>
__device__ void build_T(const bf* sK, int ldk, const float* sG, const float* sB, float* sA, float* sTf, bf* sTb, int n,
                        PhaseClock& pc, int kid) {
  wm::block_gemm<false, true>(CS, CS, KD, sK, ldk, sK, ldk, [&](int t, int s, float v) {
    sA[t * 65 + s] = (s < t && t < n) ? __expf(sG[t] - sG[s]) * v : 0.f;
  });
  for (int i = threadIdx.x; i < CS * 65; i += NT) sTf[i] = 0.f;
  __syncthreads();
  pc.mark(kid, 12);
  if (threadIdx.x < 64) {
    // diagonal blocks: each of the 4 x 16 columns of the four unit-lower 16 x 16 inverses is an
    // independent forward substitution, one thread per column with the column in registers
    const int o = (threadIdx.x >> 4) * 16, c = threadIdx.x & 15;
    float col[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < r; ++s2) acc += sA[(o + r) * 65 + o + s2] * col[s2];   // col[s2] = 0 for s2 < c
      col[r] = r < c ? 0.f : (r == c ? 1.f : -sB[o + r] * acc);
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sTf[(o + r) * 65 + o + c] = col[r];
  }
  __syncthreads();
  pc.mark(kid, 13);
  float* scratch = sTf + CS * 65;  // callers reserve 4 x 16 x 17 floats after sTf
  for (int d = 1; d < 4; ++d) {
    // the 4 - d blocks (i, j) = (j + d, j) of this level; one thread per 2 x 2 output tile (64 per
    // block), so every loaded A / T value serves two products
    const int nblk = 4 - d;
    const int j = threadIdx.x >> 6, tile = threadIdx.x & 63;
    const bool active = j < nblk;
    const int i = j + d;
    const int r0 = (tile >> 3) * 2, c0 = (tile & 7) * 2;
    float* X = scratch + (active ? j : 0) * 16 * 17;
    if (active) {
      // X = diag(beta_i) sum_{k=j}^{i-1} A_ik T_kj  (16 x 16)
      float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
      const float* ar0 = sA + (i * 16 + r0) * 65;
      const float* ar1 = ar0 + 65;
      const float* tc = sTf + j * 16 + c0;
#pragma unroll 4
      for (int m = j * 16; m < i * 16; ++m) {
        const float x0 = ar0[m], x1 = ar1[m];
        const float t0 = tc[m * 65], t1 = tc[m * 65 + 1];
        a00 += x0 * t0;
        a01 += x0 * t1;
        a10 += x1 * t0;
        a11 += x1 * t1;
      }
      const float b0 = sB[i * 16 + r0], b1 = sB[i * 16 + r0 + 1];
      X[r0 * 17 + c0] = b0 * a00;
      X[r0 * 17 + c0 + 1] = b0 * a01;
      X[(r0 + 1) * 17 + c0] = b1 * a10;
      X[(r0 + 1) * 17 + c0 + 1] = b1 * a11;
    }
    __syncthreads();
    if (active) {
      // T_ij = -T_ii X  (T_ii is zero above its diagonal)
      float a00 = 0.f, a01 = 0.f, a10 = 0.f, a11 = 0.f;
      const float* tr0 = sTf + (i * 16 + r0) * 65 + i * 16;
      const float* tr1 = tr0 + 65;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float x0 = tr0[m], x1 = tr1[m];
        const float t0 = X[m * 17 + c0], t1 = X[m * 17 + c0 + 1];
        a00 += x0 * t0;
        a01 += x0 * t1;
        a10 += x1 * t0;
        a11 += x1 * t1;
      }
      float* o0 = sTf + (i * 16 + r0) * 65 + j * 16 + c0;
      o0[0] = -a00;
      o0[1] = -a01;
      o0[65] = -a10;
      o0[66] = -a11;
    }
    __syncthreads();
  }
  pc.mark(kid, 14);
  for (int i = threadIdx.x; i < CS * CS; i += NT) {
    const int r = i / CS, c = i % CS;
    sTb[r * 72 + c] = f2b(r < n ? sTf[r * 65 + c] : 0.f);
  }
  __syncthreads();
  pc.mark(kid, 15);
}

// ------------------------------------------------------------------------------------------------ forward
template <int KD, int VD>
struct PrepSmem {
  static constexpr int LK = KD + 8, LV = VD + 8;
  static constexpr size_t K = 0;
  static constexpr size_t KB = K + sizeof(bf) * CS * LK;
  static constexpr size_t VB = KB + sizeof(bf) * CS * LK;
  static constexpr size_t A = VB + sizeof(bf) * CS * LV;
  static constexpr size_t TF = A + sizeof(float) * CS * 65;
  static constexpr size_t TB = TF + sizeof(float) * (CS * 65 + 4 * 16 * 17);   // T + blocked-inverse scratch
  static constexpr size_t VEC = TB + sizeof(bf) * CS * 72;
  static constexpr size_t TOTAL = VEC + sizeof(float) * 4 * CS;
};

template <int KD, int VD>
__global__ void __launch_bounds__(NT) gdr_prep_kernel(const bf* __restrict__ k, const bf* __restrict__ v,
                                                      const float* __restrict__ g, const float* __restrict__ beta,
                                                      const int* __restrict__ chunks, bf* __restrict__ wk,
                                                      bf* __restrict__ wv, int H) {
  using SM = PrepSmem<KD, VD>;
  extern __shared__ __align__(16) unsigned char smem[];
  bf* sK = reinterpret_cast<bf*>(smem + SM::K);
  bf* sKb = reinterpret_cast<bf*>(smem + SM::KB);
  bf* sVb = reinterpret_cast<bf*>(smem + SM::VB);
  float* sA = reinterpret_cast<float*>(smem + SM::A);
  float* sTf = reinterpret_cast<float*>(smem + SM::TF);
  bf* sTb = reinterpret_cast<bf*>(smem + SM::TB);
  float* sG = reinterpret_cast<float*>(smem + SM::VEC);
  float* sGam = sG + CS;
  float* sE = sGam + CS;
  float* sB = sE + CS;
  const Chunk ch = load_chunk_desc(chunks, blockIdx.x);
  const int h = blockIdx.y;
  PhaseClock pc;
  load_rows<KD>(sK, SM::LK, k, ch.row0, ch.n, H, h, KD, 0);
  for (int t = threadIdx.x; t < CS; t += NT) sB[t] = t < ch.n ? beta[(size_t)(ch.row0 + t) * H + h] : 0.f;
  // raw V rows into registers while the K rows are in flight
  constexpr int VPT = CS * VD / 4 / NT;
  float4 vreg[VPT];
#pragma unroll
  for (int a = 0; a < VPT; ++a) {
    const int i = threadIdx.x + a * NT;
    const int t = i / (VD / 4), c = (i % (VD / 4)) * 4;
    vreg[a] = t < ch.n ? ld_bf4(v + ((size_t)(ch.row0 + t) * H + h) * VD + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  chunk_decay(g, ch.row0, ch.n, H, h, sG, sGam, sE);
  // scaled operands: Kb = beta Gam K, Vb = beta V
#pragma unroll 4
  for (int i = threadIdx.x; i < CS * KD / 4; i += NT) {
    const int t = i / (KD / 4), c = (i % (KD / 4)) * 4;
    st_bf4(sKb + t * SM::LK + c, scale4(ld_bf4(sK + t * SM::LK + c), sB[t] * sGam[t]));
  }
#pragma unroll
  for (int a = 0; a < VPT; ++a) {
    const int i = threadIdx.x + a * NT;
    const int t = i / (VD / 4), c = (i % (VD / 4)) * 4;
    st_bf4(sVb + t * SM::LV + c, scale4(vreg[a], sB[t]));
  }
  __syncthreads();
  pc.mark(0, 0);
  build_T<KD>(sK, SM::LK, sG, sB, sA, sTf, sTb, ch.n, pc, 0);
  pc.mark(0, 1);
  // (bf16 pairs: one 4-byte store per two columns)
  wm::block_gemm_pairs<false, false>(CS, KD, CS, sTb, 72, sKb, nullptr, SM::LK, [&](int t, int c, float a, float b) {
    if (t < ch.n)
      *reinterpret_cast<__nv_bfloat162*>(wk + ((size_t)(ch.row0 + t) * H + h) * KD + c) = __floats2bfloat162_rn(a, b);
  });
  wm::block_gemm_pairs<false, false>(CS, VD, CS, sTb, 72, sVb, nullptr, SM::LV, [&](int t, int c, float a, float b) {
    if (t < ch.n)
      *reinterpret_cast<__nv_bfloat162*>(wv + ((size_t)(ch.row0 + t) * H + h) * VD + c) = __floats2bfloat162_rn(a, b);
  });
  pc.mark(0, 2);
}

template <int KD, int VB>
struct ScanSmem {
  static constexpr int LK = KD + 8, LV = VB + 8;
  // the row inputs of a chunk (Q, K, Wk, Wv), double-buffered: buffer b at ROWS * b
  static constexpr size_t Q = 0;
  static constexpr size_t K = Q + sizeof(bf) * CS * LK;
  static constexpr size_t WK = K + sizeof(bf) * CS * LK;
  static constexpr size_t WV = WK + sizeof(bf) * CS * LK;
  static constexpr size_t ROWS = WV + sizeof(bf) * CS * LV;
  static constexpr size_t S = 2 * ROWS;                        // state, bf16 hi then lo
  static constexpr size_t U = S + 2 * sizeof(bf) * KD * LV;
  static constexpr size_t EU = U + sizeof(bf) * CS * LV;
  static constexpr size_t P = EU + sizeof(bf) * CS * LV;
  static constexpr size_t VEC = P + sizeof(bf) * CS * 72;
  static constexpr size_t TOTAL = VEC + sizeof(float) * 3 * CS;
  static_assert(TOTAL <= 232448, "scan shared memory above the per-block limit");
};

// state tiles (16 x 16) of a [KD, VB] matrix owned by warp w: t = w, w + 8, ...
template <int KD, int VB>
struct StateTiles {
  static constexpr int TILES = (KD / 16) * (VB / 16);
  static constexpr int PER_WARP = (TILES + 7) / 8;
  static constexpr int TN = VB / 16;
};

template <int KD, int VD, int VB>
__global__ void __launch_bounds__(NT) gdr_scan_kernel(
    const bf* __restrict__ q, const bf* __restrict__ k, const bf* __restrict__ wk, const bf* __restrict__ wv,
    const float* __restrict__ g, const float* __restrict__ h0, const int* __restrict__ chunks,
    const int* __restrict__ seq_chunk0, bf* __restrict__ o, bf* __restrict__ u, float* __restrict__ hT,
    float* __restrict__ ckpt, int H, int nc_max, float scale) {
  using SM = ScanSmem<KD, VB>;
  using ST = StateTiles<KD, VB>;
  extern __shared__ __align__(16) unsigned char smem[];
  bf* sS = reinterpret_cast<bf*>(smem + SM::S);
  bf* sSl = sS + KD * SM::LV;
  bf* sU = reinterpret_cast<bf*>(smem + SM::U);
  bf* sEU = reinterpret_cast<bf*>(smem + SM::EU);
  bf* sP = reinterpret_cast<bf*>(smem + SM::P);
  float* sG = reinterpret_cast<float*>(smem + SM::VEC);
  float* sGam = sG + CS;
  float* sE = sGam + CS;
  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vb * VB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c_begin = seq_chunk0[b], c_end = seq_chunk0[b + 1];
  PhaseClock pc;

  float st[ST::PER_WARP][2][4];
#pragma unroll
  for (int i = 0; i < ST::PER_WARP; ++i) {
    const int t = warp + 8 * i;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = (t / ST::TN) * 16 + (lane >> 2) + 8 * (e >> 1);
        const int c = (t % ST::TN) * 16 + 8 * j + 2 * (lane & 3) + (e & 1);
        st[i][j][e] = (t < ST::TILES && h0) ? h0[(((size_t)b * H + h) * KD + r) * VD + v0 + c] : 0.f;
      }
  }
  // the next chunk's rows are fetched (cp.async) while this chunk computes
  auto fetch = [&](int cj, int buf) {
    const Chunk cn = load_chunk_desc(chunks, cj);
    unsigned char* base = smem + buf * SM::ROWS;
    load_rows<KD>(reinterpret_cast<bf*>(base + SM::Q), SM::LK, q, cn.row0, cn.n, H, h, KD, 0);
    load_rows<KD>(reinterpret_cast<bf*>(base + SM::K), SM::LK, k, cn.row0, cn.n, H, h, KD, 0);
    load_rows<KD>(reinterpret_cast<bf*>(base + SM::WK), SM::LK, wk, cn.row0, cn.n, H, h, KD, 0);
    load_rows<VB>(reinterpret_cast<bf*>(base + SM::WV), SM::LV, wv, cn.row0, cn.n, H, h, VD, v0);
    cp_async_commit();
  };
  if (c_begin < c_end) fetch(c_begin, 0);
  for (int ci = c_begin; ci < c_end; ++ci) {
    const Chunk ch = load_chunk_desc(chunks, ci);
    const int buf = (ci - c_begin) & 1;
    bf* sQ = reinterpret_cast<bf*>(smem + buf * SM::ROWS + SM::Q);
    bf* sK = reinterpret_cast<bf*>(smem + buf * SM::ROWS + SM::K);
    bf* sWk = reinterpret_cast<bf*>(smem + buf * SM::ROWS + SM::WK);
    bf* sWv = reinterpret_cast<bf*>(smem + buf * SM::ROWS + SM::WV);
    float* ck = ckpt + (((size_t)b * H + h) * nc_max + ch.c) * KD * VD;
    // checkpoint S0 (FP32) and its bf16 copy for the tensor cores
#pragma unroll
    for (int i = 0; i < ST::PER_WARP; ++i) {
      const int t = warp + 8 * i;
      if (t >= ST::TILES) continue;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = (t / ST::TN) * 16 + (lane >> 2) + 8 * (e >> 1);
          const int c = (t % ST::TN) * 16 + 8 * j + 2 * (lane & 3);
          *reinterpret_cast<float2*>(ck + (size_t)r * VD + v0 + c) = make_float2(st[i][j][e], st[i][j][e + 1]);
          wm::split_bf16(st[i][j][e], sS[r * SM::LV + c], sSl[r * SM::LV + c]);
          wm::split_bf16(st[i][j][e + 1], sS[r * SM::LV + c + 1], sSl[r * SM::LV + c + 1]);
        }
    }
    // buffer buf ^ 1 was last read by the previous chunk, which ended with a block barrier
    if (ci + 1 < c_end) {
      fetch(ci + 1, buf ^ 1);
      cp_async_wait_group<1>();   // this chunk's rows have landed; the next chunk's may still be in flight
    } else {
      cp_async_wait_group<0>();
    }
    chunk_decay<false>(g, ch.row0, ch.n, H, h, sG, sGam, sE);  // ends with __syncthreads
    pc.mark(1, 0);
    // P = D o Q K^T (s <= t)
    wm::block_gemm<false, true>(CS, CS, KD, sQ, SM::LK, sK, SM::LK, [&](int t, int s, float val) {
      sP[t * 72 + s] = f2b((s <= t && t < ch.n) ? __expf(sG[t] - sG[s]) * val : 0.f);
    });
    // U = Wv - Wk S0
    wm::block_gemm_pairs<false, false>(CS, VB, KD, sWk, SM::LK, sS, sSl, SM::LV, [&](int t, int c, float a, float b) {
      const bool ok = t < ch.n;
      const float2 wv2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sWv + t * SM::LV + c));
      const float u0 = ok ? wv2.x - a : 0.f, u1 = ok ? wv2.y - b : 0.f;
      const __nv_bfloat162 uh = __floats2bfloat162_rn(u0, u1);
      *reinterpret_cast<__nv_bfloat162*>(sU + t * SM::LV + c) = uh;
      *reinterpret_cast<__nv_bfloat162*>(sEU + t * SM::LV + c) = __floats2bfloat162_rn(sE[t] * u0, sE[t] * u1);
      if (ok) *reinterpret_cast<__nv_bfloat162*>(u + ((size_t)(ch.row0 + t) * H + h) * VD + v0 + c) = uh;
    });
    __syncthreads();
    pc.mark(1, 1);
    // O = scale (Gam o (Q S0) + P U)
    {
      const int tn = VB / 16, tiles = (CS / 16) * tn;
      for (int t = warp; t < tiles; t += 8) {
        const int m0 = (t / tn) * 16, n0 = (t % tn) * 16;
        float c1[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        float c2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        wm::warp_tile<false, false>(c1, sQ, SM::LK, sS, SM::LV, m0, n0, KD);
        wm::warp_tile<false, false>(c1, sQ, SM::LK, sSl, SM::LV, m0, n0, KD);
        wm::warp_tile<false, false>(c2, sP, 72, sU, SM::LV, m0, n0, CS);
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int r = m0 + (lane >> 2) + 8 * (e >> 1), c = n0 + 8 * j + 2 * (lane & 3);
            if (r < ch.n)
              *reinterpret_cast<__nv_bfloat162*>(o + ((size_t)(ch.row0 + r) * H + h) * VD + v0 + c) =
                  __floats2bfloat162_rn(scale * (sGam[r] * c1[j][e] + c2[j][e]),
                                        scale * (sGam[r] * c1[j][e + 1] + c2[j][e + 1]));
          }
      }
    }
    pc.mark(1, 2);
    // S1 = Gam_last S0 + K^T (E o U)
    const float gl = sGam[ch.n - 1];
#pragma unroll
    for (int i = 0; i < ST::PER_WARP; ++i) {
      const int t = warp + 8 * i;
      if (t >= ST::TILES) continue;
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      wm::warp_tile<true, false>(c, sK, SM::LK, sEU, SM::LV, (t / ST::TN) * 16, (t % ST::TN) * 16, CS);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[i][j][e] = gl * st[i][j][e] + c[j][e];
    }
    __syncthreads();
    pc.mark(1, 3);
  }
#pragma unroll
  for (int i = 0; i < ST::PER_WARP; ++i) {
    const int t = warp + 8 * i;
    if (t >= ST::TILES) continue;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = (t / ST::TN) * 16 + (lane >> 2) + 8 * (e >> 1);
        const int c = (t % ST::TN) * 16 + 8 * j + 2 * (lane & 3) + (e & 1);
        hT[(((size_t)b * H + h) * KD + r) * VD + v0 + c] = st[i][j][e];
      }
  }
}

// ------------------------------------------------------------------------------------------------ backward
template <int KD, int VB>
struct BScanSmem {
  static constexpr int LK = KD + 8, LV = VB + 8;
  // Q, K, Wk rows of a chunk, double-buffered: buffer b at ROWS * b
  static constexpr size_t Q = 0;
  static constexpr size_t K = Q + sizeof(bf) * CS * LK;
  static constexpr size_t WK = K + sizeof(bf) * CS * LK;
  static constexpr size_t ROWS = WK + sizeof(bf) * CS * LK;
  static constexpr size_t S = 2 * ROWS;
  static constexpr size_t DS = S + 2 * sizeof(bf) * KD * LV;   // S0 and dS1, each bf16 hi then lo
  static constexpr size_t U = DS + 2 * sizeof(bf) * KD * LV;
  static constexpr size_t DO = U + sizeof(bf) * CS * LV;
  static constexpr size_t GDO = DO + sizeof(bf) * CS * LV;
  static constexpr size_t NDU = GDO + sizeof(bf) * CS * LV;
  static constexpr size_t P = NDU + sizeof(bf) * CS * LV;
  static constexpr size_t VEC = P + sizeof(bf) * CS * 72;   // G Gam E dG de red
  static constexpr size_t TOTAL = VEC + sizeof(float) * (5 * CS + 32);
  static_assert(TOTAL <= 232448, "backward scan shared memory above the per-block limit");
};

template <int KD, int VD, int VB>
__global__ void __launch_bounds__(NT) gdr_bwd_scan_kernel(
    const bf* __restrict__ dout, const float* __restrict__ dhT, const bf* __restrict__ q, const bf* __restrict__ k,
    const bf* __restrict__ wk, const bf* __restrict__ u, const float* __restrict__ g, const float* __restrict__ ckpt,
    const int* __restrict__ chunks, const int* __restrict__ seq_chunk0, float* __restrict__ du,
    float* __restrict__ dwk, float* __restrict__ dq, float* __restrict__ dk, float* __restrict__ dG,
    float* __restrict__ dh0, int H, int nc_max, float scale) {
  using SM = BScanSmem<KD, VB>;
  using ST = StateTiles<KD, VB>;
  extern __shared__ __align__(16) unsigned char smem[];
  bf* sS = reinterpret_cast<bf*>(smem + SM::S);
  bf* sSl = sS + KD * SM::LV;
  bf* sdS = reinterpret_cast<bf*>(smem + SM::DS);
  bf* sdSl = sdS + KD * SM::LV;
  bf* sU = reinterpret_cast<bf*>(smem + SM::U);
  bf* sdO = reinterpret_cast<bf*>(smem + SM::DO);
  bf* sGdO = reinterpret_cast<bf*>(smem + SM::GDO);
  bf* snDU = reinterpret_cast<bf*>(smem + SM::NDU);
  bf* sP = reinterpret_cast<bf*>(smem + SM::P);
  float* sG = reinterpret_cast<float*>(smem + SM::VEC);
  float* sGam = sG + CS;
  float* sE = sGam + CS;
  float* sdG = sE + CS;
  float* sde = sdG + CS;
  float* sred = sde + CS;
  const int vb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vb * VB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c_begin = seq_chunk0[b], c_end = seq_chunk0[b + 1];
  PhaseClock pc;

  float ds[ST::PER_WARP][2][4];
#pragma unroll
  for (int i = 0; i < ST::PER_WARP; ++i) {
    const int t = warp + 8 * i;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = (t / ST::TN) * 16 + (lane >> 2) + 8 * (e >> 1);
        const int c = (t % ST::TN) * 16 + 8 * j + 2 * (lane & 3) + (e & 1);
        ds[i][j][e] = (t < ST::TILES && dhT) ? dhT[(((size_t)b * H + h) * KD + r) * VD + v0 + c] : 0.f;
      }
  }
  // Chunks run in reverse; the previous chunk's Q / K / Wk rows (cp.async, other buffer) and its FP32
  // state checkpoint (registers) are fetched while this chunk computes.
  constexpr int CPT = KD * VB / 4 / NT;   // checkpoint float4 groups per thread
  auto ck_of = [&](int cj) {
    return ckpt + (((size_t)b * H + h) * nc_max + load_chunk_desc(chunks, cj).c) * KD * VD;
  };
  auto fetch_rows = [&](int cj, int buf) {
    const Chunk cn = load_chunk_desc(chunks, cj);
    unsigned char* base = smem + buf * SM::ROWS;
    load_rows<KD>(reinterpret_cast<bf*>(base + SM::Q), SM::LK, q, cn.row0, cn.n, H, h, KD, 0);
    load_rows<KD>(reinterpret_cast<bf*>(base + SM::K), SM::LK, k, cn.row0, cn.n, H, h, KD, 0);
    load_rows<KD>(reinterpret_cast<bf*>(base + SM::WK), SM::LK, wk, cn.row0, cn.n, H, h, KD, 0);
    cp_async_commit();
  };
  float4 ckreg[CPT];
  auto fetch_ck = [&](int cj) {
    const float* src = ck_of(cj);
#pragma unroll
    for (int a = 0; a < CPT; ++a) {
      const int i = threadIdx.x + a * NT;
      const int r = i / (VB / 4), c = (i % (VB / 4)) * 4;
      ckreg[a] = *reinterpret_cast<const float4*>(src + (size_t)r * VD + v0 + c);
    }
  };
  if (c_begin < c_end) {
    fetch_rows(c_end - 1, 0);
    fetch_ck(c_end - 1);
  }
  for (int ci = c_end - 1; ci >= c_begin; --ci) {
    const Chunk ch = load_chunk_desc(chunks, ci);
    const int buf = (c_end - 1 - ci) & 1;
    bf* sQ = reinterpret_cast<bf*>(smem + buf * SM::ROWS + SM::Q);
    bf* sK = reinterpret_cast<bf*>(smem + buf * SM::ROWS + SM::K);
    bf* sWk = reinterpret_cast<bf*>(smem + buf * SM::ROWS + SM::WK);
    const float* ck = ckpt + (((size_t)b * H + h) * nc_max + ch.c) * KD * VD;
#pragma unroll
    for (int a = 0; a < CPT; ++a) {
      const int i = threadIdx.x + a * NT;
      const int r = i / (VB / 4), c = (i % (VB / 4)) * 4;
      const float4 x = ckreg[a];
      const float4 hi = ld_bf4_round(x);
      st_bf4(sS + r * SM::LV + c, hi);
      st_bf4(sSl + r * SM::LV + c, make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w));
    }
    if (ci > c_begin) fetch_ck(ci - 1);
    float dot = 0.f;  // <dS1, S0> partial
#pragma unroll
    for (int i = 0; i < ST::PER_WARP; ++i) {
      const int t = warp + 8 * i;
      if (t >= ST::TILES) continue;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = (t / ST::TN) * 16 + (lane >> 2) + 8 * (e >> 1);
          const int c = (t % ST::TN) * 16 + 8 * j + 2 * (lane & 3);
          wm::split_bf16(ds[i][j][e], sdS[r * SM::LV + c], sdSl[r * SM::LV + c]);
          wm::split_bf16(ds[i][j][e + 1], sdS[r * SM::LV + c + 1], sdSl[r * SM::LV + c + 1]);
          const float2 s0 = *reinterpret_cast<const float2*>(ck + (size_t)r * VD + v0 + c);
          dot += ds[i][j][e] * s0.x + ds[i][j][e + 1] * s0.y;
        }
    }
    dot = bb::warp_sum(dot);
    if (lane == 0) sred[warp] = dot;
    load_rows<VB>(sU, SM::LV, u, ch.row0, ch.n, H, h, VD, v0);
    load_rows<VB>(sdO, SM::LV, dout, ch.row0, ch.n, H, h, VD, v0);
    cp_async_commit();
    // buffer buf ^ 1 was last read by the chunk before, which ended with a block barrier
    if (ci > c_begin) {
      fetch_rows(ci - 1, buf ^ 1);
      cp_async_wait_group<1>();   // this chunk's rows (and U / dO) have landed
    } else {
      cp_async_wait_group<0>();
    }
    for (int t = threadIdx.x; t < CS; t += NT) sdG[t] = sde[t] = 0.f;
    chunk_decay<false>(g, ch.row0, ch.n, H, h, sG, sGam, sE);  // syncs
    for (int i = threadIdx.x; i < CS * VB; i += NT) {
      const int t = i / VB, c = i % VB;
      sGdO[t * SM::LV + c] = f2b(scale * sGam[t] * b2f(sdO[t * SM::LV + c]));
    }
    pc.mark(2, 0);
    wm::block_gemm<false, true>(CS, CS, KD, sQ, SM::LK, sK, SM::LK, [&](int t, int s, float val) {
      sP[t * 72 + s] = f2b((s <= t && t < ch.n) ? __expf(sG[t] - sG[s]) * val : 0.f);
    });
    __syncthreads();
    pc.mark(2, 1);
    // dU = scale P^T dO + E o (K dS1);  de_s = sum_j (K dS1)_sj U_sj
    {
      const int tn = VB / 16, tiles = (CS / 16) * tn;
      for (int t = warp; t < tiles; t += 8) {
        const int m0 = (t / tn) * 16, n0 = (t % tn) * 16;
        float c1[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        float c2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        wm::warp_tile<false, false>(c1, sK, SM::LK, sdS, SM::LV, m0, n0, KD);
        wm::warp_tile<false, false>(c1, sK, SM::LK, sdSl, SM::LV, m0, n0, KD);
        wm::warp_tile<true, false>(c2, sP, 72, sdO, SM::LV, m0, n0, CS);
        float racc[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int r = m0 + (lane >> 2) + 8 * (e >> 1), c = n0 + 8 * j + 2 * (lane & 3);
            const bool ok = r < ch.n;
            const float d0 = ok ? scale * c2[j][e] + sE[r] * c1[j][e] : 0.f;
            const float d1 = ok ? scale * c2[j][e + 1] + sE[r] * c1[j][e + 1] : 0.f;
            *reinterpret_cast<__nv_bfloat162*>(snDU + r * SM::LV + c) = __floats2bfloat162_rn(-d0, -d1);
            if (ok) {
              *reinterpret_cast<float2*>(du + ((size_t)(ch.row0 + r) * H + h) * VD + v0 + c) = make_float2(d0, d1);
              const float2 uu = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sU + r * SM::LV + c));
              racc[e >> 1] += c1[j][e] * uu.x + c1[j][e + 1] * uu.y;
            }
          }
        // per-row sums inside the tile first (four lanes share a row), one shared atomic per row
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float v = racc[hh];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          if ((lane & 3) == 0 && v != 0.f) atomicAdd(&sde[m0 + (lane >> 2) + 8 * hh], v);
        }
      }
    }
    __syncthreads();
    pc.mark(2, 2);
    // state-dependent gradient pieces (summed over the V blocks with atomics)
    // (float2 atomics: the two V blocks of a head add into the same rows)
    wm::block_gemm_pairs<false, true>(CS, KD, VB, sdO, SM::LV, sS, sSl, SM::LV, [&](int t, int c, float a, float b) {
      if (t < ch.n) {
        const float f = scale * sGam[t];
        atomicAdd(reinterpret_cast<float2*>(&dq[((size_t)(ch.row0 + t) * H + h) * KD + c]), make_float2(f * a, f * b));
      }
    });
    pc.mark(2, 3);
    wm::block_gemm_pairs<false, true>(CS, KD, VB, sU, SM::LV, sdS, sdSl, SM::LV, [&](int t, int c, float a, float b) {
      if (t < ch.n)
        atomicAdd(reinterpret_cast<float2*>(&dk[((size_t)(ch.row0 + t) * H + h) * KD + c]),
                  make_float2(sE[t] * a, sE[t] * b));
    });
    pc.mark(2, 4);
    wm::block_gemm_pairs<false, true>(CS, KD, VB, snDU, SM::LV, sS, sSl, SM::LV, [&](int t, int c, float a, float b) {
      if (t < ch.n) atomicAdd(reinterpret_cast<float2*>(&dwk[((size_t)(ch.row0 + t) * H + h) * KD + c]), make_float2(a, b));
    });
    pc.mark(2, 5);
    wm::block_gemm_red<false, false>(CS, VB, KD, sQ, SM::LK, sS, sSl, SM::LV, sdG, nullptr, nullptr,
                                     [&](int t, int c, float val, float (&rc)[2], float (&)[1]) {
      if (t < ch.n) rc[0] += scale * sGam[t] * val * b2f(sdO[t * SM::LV + c]);
    });
    pc.mark(2, 6);
    // dS0 = Gam_last dS1 + Q^T (scale Gam o dO) - Wk^T dU
    const float gl = sGam[ch.n - 1];
#pragma unroll
    for (int i = 0; i < ST::PER_WARP; ++i) {
      const int t = warp + 8 * i;
      if (t >= ST::TILES) continue;
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const int m0 = (t / ST::TN) * 16, n0 = (t % ST::TN) * 16;
      wm::warp_tile<true, false>(c, sQ, SM::LK, sGdO, SM::LV, m0, n0, CS);
      wm::warp_tile<true, false>(c, sWk, SM::LK, snDU, SM::LV, m0, n0, CS);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) ds[i][j][e] = gl * ds[i][j][e] + c[j][e];
    }
    __syncthreads();
    pc.mark(2, 7);
    if (threadIdx.x == 0) {
      float tot = 0.f, dsum = 0.f;
      for (int w = 0; w < NT / 32; ++w) dsum += sred[w];
      for (int t = 0; t < ch.n; ++t) tot += sde[t] * sE[t];
      sdG[ch.n - 1] += dsum * gl + tot;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < ch.n; t += NT)
      atomicAdd(&dG[(size_t)(ch.row0 + t) * H + h], sdG[t] - sde[t] * sE[t]);
    __syncthreads();
    pc.mark(2, 8);
  }
  if (dh0) {
#pragma unroll
    for (int i = 0; i < ST::PER_WARP; ++i) {
      const int t = warp + 8 * i;
      if (t >= ST::TILES) continue;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = (t / ST::TN) * 16 + (lane >> 2) + 8 * (e >> 1);
          const int c = (t % ST::TN) * 16 + 8 * j + 2 * (lane & 3) + (e & 1);
          dh0[(((size_t)b * H + h) * KD + r) * VD + v0 + c] = ds[i][j][e];
        }
    }
  }
}

template <int KD, int VD>
struct BChunkSmem {
  static constexpr int LK = KD + 8, LV = VD + 8;
  static constexpr size_t Q = 0;
  static constexpr size_t K = Q + sizeof(bf) * CS * LK;
  static constexpr size_t KB = K + sizeof(bf) * CS * LK;
  static constexpr size_t DWK = KB + sizeof(bf) * CS * LK;
  static constexpr size_t U = DWK + sizeof(bf) * CS * LK;
  static constexpr size_t DO = U + sizeof(bf) * CS * LV;
  static constexpr size_t DU = DO + sizeof(bf) * CS * LV;
  static constexpr size_t VB = DU + sizeof(bf) * CS * LV;
  static constexpr size_t TB = VB + sizeof(bf) * CS * LV;
  static constexpr size_t X1 = TB + sizeof(bf) * CS * 72;   // dP o D, then dT / M
  static constexpr size_t X2 = X1 + sizeof(bf) * CS * 72;   // dT T^T
  static constexpr size_t A = X2 + sizeof(bf) * CS * 72;
  static constexpr size_t TF = A + sizeof(float) * CS * 65;  // T (solve) + scratch, then P
  static constexpr size_t VEC = TF + sizeof(float) * (CS * 65 + 4 * 16 * 17);  // G Gam E B dG db
  static constexpr size_t TOTAL = VEC + sizeof(float) * 6 * CS;
  // from the dq / dk phase on, U and dO are dead: their bytes hold the FP32 dk accumulator [64][KD + 4]
  static constexpr int LDK = KD + 4;
  static_assert(DO == U + sizeof(bf) * CS * LV && sizeof(float) * CS * LDK <= 2 * sizeof(bf) * CS * LV,
                "dk accumulator must fit in the U + dO buffers");
};

template <int KD, int VD>
__global__ void __launch_bounds__(NT) gdr_bwd_chunk_kernel(
    const bf* __restrict__ dout, const bf* __restrict__ q, const bf* __restrict__ k, const bf* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, const bf* __restrict__ u,
    const float* __restrict__ du, const float* __restrict__ dwk, const int* __restrict__ chunks,
    float* __restrict__ dq, float* __restrict__ dk, bf* __restrict__ dv, const float* __restrict__ dG_in,
    float* __restrict__ dg, float* __restrict__ dbeta, int H, float scale) {
  using SM = BChunkSmem<KD, VD>;
  extern __shared__ __align__(16) unsigned char smem[];
  bf* sQ = reinterpret_cast<bf*>(smem + SM::Q);
  bf* sK = reinterpret_cast<bf*>(smem + SM::K);
  bf* sKb = reinterpret_cast<bf*>(smem + SM::KB);
  bf* sdWk = reinterpret_cast<bf*>(smem + SM::DWK);
  bf* sU = reinterpret_cast<bf*>(smem + SM::U);
  bf* sdO = reinterpret_cast<bf*>(smem + SM::DO);
  bf* sdU = reinterpret_cast<bf*>(smem + SM::DU);
  bf* sVb = reinterpret_cast<bf*>(smem + SM::VB);
  bf* sTb = reinterpret_cast<bf*>(smem + SM::TB);
  bf* sX1 = reinterpret_cast<bf*>(smem + SM::X1);
  bf* sX2 = reinterpret_cast<bf*>(smem + SM::X2);
  float* sA = reinterpret_cast<float*>(smem + SM::A);
  float* sTf = reinterpret_cast<float*>(smem + SM::TF);
  float* sG = reinterpret_cast<float*>(smem + SM::VEC);
  float* sGam = sG + CS;
  float* sE = sGam + CS;
  float* sB = sE + CS;
  float* sdG = sB + CS;
  float* sdb = sdG + CS;
  const Chunk ch = load_chunk_desc(chunks, blockIdx.x);
  const int h = blockIdx.y, n = ch.n, row0 = ch.row0;
  PhaseClock pc;
  auto rk = [&](int t) { return ((size_t)(row0 + t) * H + h) * KD; };
  auto rv = [&](int t) { return ((size_t)(row0 + t) * H + h) * VD; };

  load_rows<KD>(sQ, SM::LK, q, row0, n, H, h, KD, 0);
  load_rows<KD>(sK, SM::LK, k, row0, n, H, h, KD, 0);
  load_rows<VD>(sU, SM::LV, u, row0, n, H, h, VD, 0);
  load_rows<VD>(sdO, SM::LV, dout, row0, n, H, h, VD, 0);
  for (int t = threadIdx.x; t < CS; t += NT) {
    sB[t] = t < n ? beta[(size_t)(row0 + t) * H + h] : 0.f;
    sdG[t] = t < n ? dG_in[(size_t)(row0 + t) * H + h] : 0.f;
    sdb[t] = 0.f;
  }
  // the FP32 dWk / dU rows and the raw V rows are read while the cp.async rows are in flight (V is
  // held in registers until beta is visible)
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int i = threadIdx.x; i < CS * KD / 4; i += NT) {
    const int t = i / (KD / 4), c = (i % (KD / 4)) * 4;
    st_bf4(sdWk + t * SM::LK + c, t < n ? *reinterpret_cast<const float4*>(dwk + rk(t) + c) : z4);
  }
  constexpr int VPT = CS * VD / 4 / NT;   // V float4 groups per thread
  float4 vreg[VPT];
#pragma unroll
  for (int a = 0; a < VPT; ++a) {
    const int i = threadIdx.x + a * NT;
    const int t = i / (VD / 4), c = (i % (VD / 4)) * 4;
    st_bf4(sdU + t * SM::LV + c, t < n ? *reinterpret_cast<const float4*>(du + rv(t) + c) : z4);
    vreg[a] = t < n ? ld_bf4(v + rv(t) + c) : z4;
  }
  chunk_decay(g, row0, n, H, h, sG, sGam, sE);
#pragma unroll 4
  for (int i = threadIdx.x; i < CS * KD / 4; i += NT) {
    const int t = i / (KD / 4), c = (i % (KD / 4)) * 4;
    st_bf4(sKb + t * SM::LK + c, scale4(ld_bf4(sK + t * SM::LK + c), sB[t] * sGam[t]));
  }
#pragma unroll
  for (int a = 0; a < VPT; ++a) {
    const int i = threadIdx.x + a * NT;
    const int t = i / (VD / 4), c = (i % (VD / 4)) * 4;
    st_bf4(sVb + t * SM::LV + c, scale4(vreg[a], sB[t]));
  }
  __syncthreads();
  pc.mark(3, 0);
  build_T<KD>(sK, SM::LK, sG, sB, sA, sTf, sTb, n, pc, 3);   // sA = D o KK^T (strict), sTb = T
  pc.mark(3, 1);
  // P (fp32, into sTf) and dP = scale dO U^T;  dG from P: rowsum(dP o P) - colsum(dP o P)
  wm::block_gemm<false, true>(CS, CS, KD, sQ, SM::LK, sK, SM::LK, [&](int t, int s, float val) {
    sTf[t * 65 + s] = (s <= t && t < n) ? __expf(sG[t] - sG[s]) * val : 0.f;
  });
  __syncthreads();
  pc.mark(3, 2);
  wm::block_gemm_red<false, true>(CS, CS, VD, sdO, SM::LV, sU, nullptr, SM::LV, sdG, nullptr, sdG,
                                  [&](int t, int s, float val, float (&rc)[2], float (&cc)[1]) {
    const bool ok = s <= t && t < n;
    const float dp = ok ? scale * val : 0.f;
    sX1[t * 72 + s] = f2b(ok ? dp * __expf(sG[t] - sG[s]) : 0.f);
    if (ok && s != t) {
      const float pp = dp * sTf[t * 65 + s];
      rc[0] += pp;
      cc[0] -= pp;
    }
  });
  __syncthreads();
  pc.mark(3, 3);
  // dq += (dP o D) K ;  dk += (dP o D)^T Q
  // (float2 atomics whose result is unused: the add is posted, the warp does not wait for the old value)
  wm::block_gemm_pairs<false, false>(CS, KD, CS, sX1, 72, sK, nullptr, SM::LK, [&](int t, int c, float a, float b) {
    if (t < n) atomicAdd(reinterpret_cast<float2*>(dq + rk(t) + c), make_float2(a, b));
  });
  // the in-chunk dk terms are summed in shared memory (dead U / dO bytes) and added to dk once at the end
  float* sDK = reinterpret_cast<float*>(smem + SM::U);
  wm::block_gemm<true, false>(CS, KD, CS, sX1, 72, sQ, SM::LK, [&](int t, int c, float val) {
    sDK[t * SM::LDK + c] = val;
  });
  __syncthreads();
  // raw V rows (for dbeta) into the now dead Q buffer when they fit, in flight during dT
  constexpr bool kVInQ = VD <= SM::LK;
  if (kVInQ) load_rows<VD>(sQ, SM::LK, v, row0, n, H, h, VD, 0);
  pc.mark(3, 4);
  // dT = dU (beta V)^T + dWk (beta Gam K)^T   (into sX1)
  {
    const int tiles = (CS / 16) * (CS / 16);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < tiles; t += 8) {
      const int m0 = (t / 4) * 16, n0 = (t % 4) * 16;
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      wm::warp_tile<false, true>(c, sdU, SM::LV, sVb, SM::LV, m0, n0, VD);
      wm::warp_tile<false, true>(c, sdWk, SM::LK, sKb, SM::LK, m0, n0, KD);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = m0 + (lane >> 2) + 8 * (e >> 1), cc = n0 + 8 * j + 2 * (lane & 3) + (e & 1);
          sX1[r * 72 + cc] = f2b(r < n && cc < n ? c[j][e] : 0.f);
        }
    }
  }
  cp_async_wait_all();
  __syncthreads();
  pc.mark(3, 5);
  // dVb = T^T dU -> dv = beta dVb, dbeta += <dVb, V>;  dKb = T^T dWk -> dk += beta Gam dKb, dbeta, dG
  wm::block_gemm_red<true, false>(CS, VD, CS, sTb, 72, sdU, nullptr, SM::LV, sdb, nullptr, nullptr,
                                  [&](int s, int c, float val, float (&rc)[2], float (&)[1]) {
    if (s < n) {
      dv[rv(s) + c] = f2b(sB[s] * val);
      rc[0] += val * (kVInQ ? b2f(sQ[s * SM::LK + c]) : b2f(v[rv(s) + c]));
    }
  });
  wm::block_gemm_red<true, false>(CS, KD, CS, sTb, 72, sdWk, nullptr, SM::LK, sdb, sdG, nullptr,
                                  [&](int s, int c, float val, float (&rc)[2], float (&)[1]) {
    if (s < n) {
      const float kv = b2f(sK[s * SM::LK + c]);
      sDK[s * SM::LDK + c] += sB[s] * sGam[s] * val;
      rc[0] += sGam[s] * kv * val;
      rc[1] += sB[s] * sGam[s] * kv * val;
    }
  });
  pc.mark(3, 6);
  // X2 = dT T^T
  wm::block_gemm<false, true>(CS, CS, CS, sX1, 72, sTb, 72, [&](int t, int s, float val) {
    sX2[t * 72 + s] = f2b(val);
  });
  __syncthreads();
  pc.mark(3, 7);
  for (int i = threadIdx.x; i < CS * 72; i += NT) sX1[i] = f2b(0.f);
  __syncthreads();
  // dL = -T^T X2;  dA_ts = beta_t dL_ts (s < t) -> dbeta, dG, and M = dKK + dKK^T with dKK = dA o D
  wm::block_gemm_red<true, false>(CS, CS, CS, sTb, 72, sX2, nullptr, 72, sdb, sdG, sdG,
                                  [&](int t, int s, float val, float (&rc)[2], float (&cc)[1]) {
    if (s < t && t < n) {
      const float dl = -val;
      const float a = sA[t * 65 + s];
      const float da = sB[t] * dl;
      rc[0] += dl * a;
      rc[1] += da * a;
      cc[0] -= da * a;
      const bf m = f2b(da * __expf(sG[t] - sG[s]));
      sX1[t * 72 + s] = m;
      sX1[s * 72 + t] = m;
    }
  });
  __syncthreads();
  pc.mark(3, 8);
  wm::block_gemm<false, false>(CS, KD, CS, sX1, 72, sK, SM::LK, [&](int t, int c, float val) {
    sDK[t * SM::LDK + c] += val;
  });
  __syncthreads();
  // one coalesced pass of posted float4 adds into dk (the scan kernel already added the state terms)
  for (int i = threadIdx.x; i < CS * (KD / 4); i += NT) {
    const int t = i / (KD / 4), c4 = (i % (KD / 4)) * 4;
    if (t < n) {
      const float* src = sDK + t * SM::LDK + c4;
      atomicAdd(reinterpret_cast<float4*>(dk + rk(t) + c4), make_float4(src[0], src[1], src[2], src[3]));
    }
  }
  pc.mark(3, 9);
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int t = n - 1; t >= 0; --t) {
      acc += sdG[t];
      dg[(size_t)(row0 + t) * H + h] = acc;
      dbeta[(size_t)(row0 + t) * H + h] = sdb[t];
    }
  }
  pc.mark(3, 10);
}

template <typename Kern>
void set_smem(Kern kern, size_t bytes) {
  BB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

template <int KD, int VD>
void launch_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& g,
                const torch::Tensor& beta, const float* h0, const torch::Tensor& chunks, const torch::Tensor& seq0,
                torch::Tensor& o, torch::Tensor& u, torch::Tensor& hT, torch::Tensor& ckpt, torch::Tensor& wk,
                torch::Tensor& wv, int H, int B, int nct, int nc_max, float scale) {
  constexpr int VB = VD > 64 ? 64 : VD;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto prep = gdr_prep_kernel<KD, VD>;
  set_smem(prep, PrepSmem<KD, VD>::TOTAL);
  prep<<<dim3(nct, H), NT, PrepSmem<KD, VD>::TOTAL, stream>>>(
      (const bf*)k.data_ptr(), (const bf*)v.data_ptr(), g.data_ptr<float>(), beta.data_ptr<float>(),
      chunks.data_ptr<int>(), (bf*)wk.data_ptr(), (bf*)wv.data_ptr(), H);
  BB_POST_LAUNCH();
  auto scan = gdr_scan_kernel<KD, VD, VB>;
  set_smem(scan, ScanSmem<KD, VB>::TOTAL);
  scan<<<dim3(VD / VB, H, B), NT, ScanSmem<KD, VB>::TOTAL, stream>>>(
      (const bf*)q.data_ptr(), (const bf*)k.data_ptr(), (const bf*)wk.data_ptr(), (const bf*)wv.data_ptr(),
      g.data_ptr<float>(), h0, chunks.data_ptr<int>(), seq0.data_ptr<int>(), (bf*)o.data_ptr(), (bf*)u.data_ptr(),
      hT.data_ptr<float>(), ckpt.data_ptr<float>(), H, nc_max, scale);
  BB_POST_LAUNCH();
}

template <int KD, int VD>
void launch_bwd(const torch::Tensor& dout, const float* dhT, const torch::Tensor& q, const torch::Tensor& k,
                const torch::Tensor& v, const torch::Tensor& g, const torch::Tensor& beta, const torch::Tensor& ckpt,
                const torch::Tensor& wk, const torch::Tensor& u, const torch::Tensor& chunks,
                const torch::Tensor& seq0, torch::Tensor& du, torch::Tensor& dwk, torch::Tensor& dq,
                torch::Tensor& dk, torch::Tensor& dv, torch::Tensor& dG, torch::Tensor& dg, torch::Tensor& db,
                float* dh0, int H, int B, int nct, int nc_max, float scale) {
  constexpr int VB = VD > 64 ? 64 : VD;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto scan = gdr_bwd_scan_kernel<KD, VD, VB>;
  set_smem(scan, BScanSmem<KD, VB>::TOTAL);
  scan<<<dim3(VD / VB, H, B), NT, BScanSmem<KD, VB>::TOTAL, stream>>>(
      (const bf*)dout.data_ptr(), dhT, (const bf*)q.data_ptr(), (const bf*)k.data_ptr(), (const bf*)wk.data_ptr(),
      (const bf*)u.data_ptr(), g.data_ptr<float>(), ckpt.data_ptr<float>(), chunks.data_ptr<int>(),
      seq0.data_ptr<int>(), du.data_ptr<float>(), dwk.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr<float>(),
      dG.data_ptr<float>(), dh0, H, nc_max, scale);
  BB_POST_LAUNCH();
  auto chunk = gdr_bwd_chunk_kernel<KD, VD>;
  set_smem(chunk, BChunkSmem<KD, VD>::TOTAL);
  chunk<<<dim3(nct, H), NT, BChunkSmem<KD, VD>::TOTAL, stream>>>(
      (const bf*)dout.data_ptr(), (const bf*)q.data_ptr(), (const bf*)k.data_ptr(), (const bf*)v.data_ptr(),
      g.data_ptr<float>(), beta.data_ptr<float>(), (const bf*)u.data_ptr(), du.data_ptr<float>(),
      dwk.data_ptr<float>(), chunks.data_ptr<int>(), dq.data_ptr<float>(), dk.data_ptr<float>(), (bf*)dv.data_ptr(),
      dG.data_ptr<float>(), dg.data_ptr<float>(), db.data_ptr<float>(), H, scale);
  BB_POST_LAUNCH();
}

}  // namespace

// Phase timing of the gated-delta-rule kernels (a profiling aid; see PhaseClock).  Enabling clears
// the table; reading returns int64 [4, 16] summed SM cycles per (kernel, phase).
void gdr_phase_profile(bool enable) {
  const int on = enable ? 1 : 0;
  unsigned long long zero[4][16] = {};
  BB_CHECK_CUDA(cudaMemcpyToSymbol(g_gdr_prof, zero, sizeof(zero)));
  BB_CHECK_CUDA(cudaMemcpyToSymbol(g_gdr_prof_on, &on, sizeof(on)));
}

torch::Tensor gdr_phase_read() {
  unsigned long long tab[4][16];
  BB_CHECK_CUDA(cudaMemcpyFromSymbol(tab, g_gdr_prof, sizeof(tab)));
  auto out = torch::empty({4, 16}, torch::TensorOptions().dtype(torch::kInt64));
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 16; ++j) out[i][j] = (int64_t)tab[i][j];
  return out;
}

namespace {

#define BB_GDR_DISPATCH(KD, VD, CALL)                                                  \
  if (K == KD && V == VD) {                                                           \
    CALL;                                                                             \
    done = true;                                                                      \
  }

}  // namespace

// chunks: int32 [nct, 4] = (row0, n, sequence, chunk index within the sequence); seq0: int32 [B+1] first
// chunk of every sequence.  Returns {o, hT, ckpt, wk, u}.
std::vector<torch::Tensor> gdr_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                   torch::Tensor beta, c10::optional<torch::Tensor> h0, torch::Tensor chunks,
                                   torch::Tensor seq0, int64_t max_chunks, double scale) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
              "gdr: q/k/v contiguous bf16");
  TORCH_CHECK(g.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat && g.is_contiguous() &&
                  beta.is_contiguous(), "gdr: g / beta fp32 contiguous");
  const int T = q.size(0), H = q.size(1), K = q.size(2), V = v.size(2);
  const int B = seq0.numel() - 1, nct = chunks.size(0), ncm = std::max<int>(1, (int)max_chunks);
  auto o = torch::empty_like(v);
  auto u = torch::empty_like(v);
  auto wk = torch::empty_like(k);
  auto wv = torch::empty_like(v);
  auto hT = torch::empty({B, H, K, V}, q.options().dtype(at::kFloat));
  auto ckpt = torch::empty({B, H, ncm, K, V}, q.options().dtype(at::kFloat));
  torch::Tensor h0f;
  if (h0.has_value()) h0f = h0->to(at::kFloat).contiguous();
  if (T == 0 || B == 0) {
    if (h0.has_value()) hT.copy_(h0f);
    else hT.zero_();
    return {o, hT, ckpt, wk, u};
  }
  const float* h0p = h0.has_value() ? h0f.data_ptr<float>() : nullptr;
  bool done = false;
  const float sc = (float)scale;
  BB_GDR_DISPATCH(128, 128, (launch_fwd<128, 128>(q, k, v, g, beta, h0p, chunks, seq0, o, u, hT, ckpt, wk, wv, H, B, nct, ncm, sc)))
  BB_GDR_DISPATCH(64, 64, (launch_fwd<64, 64>(q, k, v, g, beta, h0p, chunks, seq0, o, u, hT, ckpt, wk, wv, H, B, nct, ncm, sc)))
  BB_GDR_DISPATCH(32, 64, (launch_fwd<32, 64>(q, k, v, g, beta, h0p, chunks, seq0, o, u, hT, ckpt, wk, wv, H, B, nct, ncm, sc)))
  BB_GDR_DISPATCH(64, 128, (launch_fwd<64, 128>(q, k, v, g, beta, h0p, chunks, seq0, o, u, hT, ckpt, wk, wv, H, B, nct, ncm, sc)))
  BB_GDR_DISPATCH(32, 32, (launch_fwd<32, 32>(q, k, v, g, beta, h0p, chunks, seq0, o, u, hT, ckpt, wk, wv, H, B, nct, ncm, sc)))
  TORCH_CHECK(done, "gdr: unsupported (key dim, value dim) = (", K, ", ", V, ")");
  return {o, hT, ckpt, wk, u};
}

std::vector<torch::Tensor> gdr_bwd(torch::Tensor dout, c10::optional<torch::Tensor> dhT, torch::Tensor q,
                                   torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                                   torch::Tensor ckpt, torch::Tensor wk, torch::Tensor u, torch::Tensor chunks,
                                   torch::Tensor seq0, int64_t max_chunks, bool has_h0, double scale) {
  const int T = q.size(0), H = q.size(1), K = q.size(2), V = v.size(2);
  const int B = seq0.numel() - 1, nct = chunks.size(0), ncm = std::max<int>(1, (int)max_chunks);
  auto f32 = q.options().dtype(at::kFloat);
  auto dq = torch::zeros({T, H, K}, f32);
  auto dk = torch::zeros({T, H, K}, f32);
  auto dv = torch::empty_like(v);
  auto dg = torch::zeros({T, H}, f32);
  auto db = torch::zeros({T, H}, f32);
  auto dh0 = torch::zeros({B, H, K, V}, f32);
  if (T == 0 || B == 0) {
    if (has_h0 && dhT.has_value()) dh0.copy_(*dhT);
    return {dq, dk, dv, dg, db, dh0};
  }
  auto du = torch::empty({T, H, V}, f32);
  auto dwk = torch::zeros({T, H, K}, f32);
  auto dG = torch::zeros({T, H}, f32);
  auto doc = dout.contiguous();
  torch::Tensor dhTf;
  if (dhT.has_value()) dhTf = dhT->to(at::kFloat).contiguous();
  const float* dhTp = dhT.has_value() ? dhTf.data_ptr<float>() : nullptr;
  float* dh0p = has_h0 ? dh0.data_ptr<float>() : nullptr;
  bool done = false;
  const float sc = (float)scale;
#define BB_B(KD, VD) launch_bwd<KD, VD>(doc, dhTp, q, k, v, g, beta, ckpt, wk, u, chunks, seq0, du, dwk, dq, dk, dv, dG, dg, db, dh0p, H, B, nct, ncm, sc)
  BB_GDR_DISPATCH(128, 128, BB_B(128, 128))
  BB_GDR_DISPATCH(64, 64, BB_B(64, 64))
  BB_GDR_DISPATCH(32, 64, BB_B(32, 64))
  BB_GDR_DISPATCH(64, 128, BB_B(64, 128))
  BB_GDR_DISPATCH(32, 32, BB_B(32, 32))
#undef BB_B
  TORCH_CHECK(done, "gdr: unsupported (key dim, value dim) = (", K, ", ", V, ")");
  return {dq, dk, dv, dg, db, dh0};
}
