// Tree (prefix-reuse) flash attention, forward and backward, bf16 in / FP32 statistics.
//
// Packed layout: q [T, Hq, D], k/v [T, Hkv, D] (own tokens), pk/pv [P, Hkv, D] (prefix bank).
// Sequence b owns rows cu[b]..cu[b+1] and sees bank rows [poff[b], poff[b]+plen[b]) fully plus its
// own rows causally.  GQA: q head h reads kv head h / (Hq/Hkv).
//
// Forward: one CTA = 64 query rows x 1 q head, 4 warps x 16 rows, KV tiles of 64 keys double
// buffered with cp.async; online softmax in FP32 (exp2 domain); writes O (bf16) and LSE [Hq, T].
//
// Backward: one CTA = 64 keys x 1 kv head; it loops over every (q head of the GQA group, q tile)
// that sees its keys and accumulates dK/dV in registers -- for a PREFIX tile that is every query
// row of every sequence reading the span (the CSR "users" list), so the shared-prefix gradient of
// all siblings is reduced here, once, without atomics.  dQ is accumulated with FP32 atomics.
//
// Tensor-core path: mma.sync m16n8k16 (bf16 -> fp32) fed by ldmatrix from padded shared memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace {

constexpr int BM = 64;  // query rows per tile
constexpr int BN = 64;  // keys per tile
constexpr int NWARP = 4;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int D>
struct Smem {
  static constexpr int LD = D + 8;  // padded row (halves): rows land in different banks for ldmatrix
};

// Load a [64 x D] tile: rows r -> gmem row pointer given by `rowptr(r)` (nullptr -> zero fill).
template <int D, typename RowPtr>
__device__ __forceinline__ void load_tile(__nv_bfloat16* s, RowPtr rowptr, const __nv_bfloat16* fallback) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
  for (int i = threadIdx.x; i < 64 * CH; i += NWARP * 32) {
    const int r = i / CH, c = i % CH;
    const __nv_bfloat16* g = rowptr(r);
    cp_async16(s + r * Smem<D>::LD + c * 8, g ? g + c * 8 : fallback, g != nullptr);
  }
}

// ================================================================================= forward
template <int D>
__global__ void __launch_bounds__(NWARP * 32) tree_attn_fwd_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const __nv_bfloat16* __restrict__ pk, const __nv_bfloat16* __restrict__ pv, const int* __restrict__ cu,
    const int* __restrict__ poff, const int* __restrict__ plen, __nv_bfloat16* __restrict__ o,
    float* __restrict__ lse, int T, int Hq, int Hk, float scale_log2) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int LD = Smem<D>::LD;
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sK = sQ + BM * LD;          // 2 stages
  __nv_bfloat16* sV = sK + 2 * BN * LD;      // 2 stages

  const int seq = blockIdx.y, h = blockIdx.z, hk = h / (Hq / Hk);
  const int q0 = cu[seq], n = cu[seq + 1] - q0;
  const int m0 = blockIdx.x * BM;
  if (m0 >= n) return;
  const int po = poff[seq], pl = plen[seq];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;

  const size_t qstride = (size_t)Hq * D, kstride = (size_t)Hk * D;
  load_tile<D>(sQ, [&](int r) -> const __nv_bfloat16* {
    return (m0 + r < n) ? q + (size_t)(q0 + m0 + r) * qstride + (size_t)h * D : nullptr;
  }, q);
  const int nkeys = pl + min(n, m0 + BM);  // keys any row of this tile can see
  const int ntiles = (nkeys + BN - 1) / BN;
  auto key_row = [&](const __nv_bfloat16* own, const __nv_bfloat16* bank, int j) -> const __nv_bfloat16* {
    if (j >= nkeys) return nullptr;
    if (j < pl) return bank + (size_t)(po + j) * kstride + (size_t)hk * D;
    return own + (size_t)(q0 + j - pl) * kstride + (size_t)hk * D;
  };
  load_tile<D>(sK, [&](int r) { return key_row(k, pk, r); }, k);
  load_tile<D>(sV, [&](int r) { return key_row(v, pv, r); }, v);
  cp_async_commit();

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int qr0 = m0 + warp * 16 + g;  // local query indices of this thread's two rows
  const int qr1 = qr0 + 8;

  for (int t = 0; t < ntiles; ++t) {
    const int stage = t & 1;
    if (t + 1 < ntiles) {
      const int kb = (t + 1) * BN;
      __nv_bfloat16* dK = sK + (stage ^ 1) * BN * LD;
      __nv_bfloat16* dV = sV + (stage ^ 1) * BN * LD;
      load_tile<D>(dK, [&](int r) { return key_row(k, pk, kb + r); }, k);
      load_tile<D>(dV, [&](int r) { return key_row(v, pv, kb + r); }, v);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* cK = sK + stage * BN * LD;
    const __nv_bfloat16* cV = sV + stage * BN * LD;

    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[4];
      ldsm_x4(a[0], a[1], a[2], a[3], sQ + (warp * 16 + (lane & 15)) * LD + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3,
                cK + (np * 16 + (lane & 7) + (lane >> 4) * 8) * LD + ks * 16 + ((lane >> 3) & 1) * 8);
        mma16816(s[2 * np], a, b0, b1);
        mma16816(s[2 * np + 1], a, b2, b3);
      }
    }
    // mask + online softmax (exp2 domain)
    const int kb = t * BN;
    float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = kb + nt * 8 + tig * 2 + (e & 1);
        const int qr = (e < 2) ? qr0 : qr1;
        bool ok = j < nkeys && (j < pl || (j - pl) <= qr) && qr < n;
        float x = ok ? s[nt][e] * scale_log2 : -INFINITY;
        s[nt][e] = x;
        mnew[e >> 1] = fmaxf(mnew[e >> 1], x);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 1));
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 2));
    }
    float alpha[2], msafe[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      msafe[r] = (mnew[r] == -INFINITY) ? 0.f : mnew[r];
      alpha[r] = exp2f(mrow[r] - msafe[r]);
      mrow[r] = mnew[r];
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float p = exp2f(s[nt][e] - msafe[e >> 1]);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * alpha[r] + rs[r];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      acc[i][0] *= alpha[0];
      acc[i][1] *= alpha[0];
      acc[i][2] *= alpha[1];
      acc[i][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3, cV + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + dp * 16 + (lane >> 4) * 8);
        mma16816(acc[2 * dp], a, b0, b1);
        mma16816(acc[2 * dp + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f;
  const float inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
  const float LN2 = 0.6931471805599453f;
  if (qr0 < n) {
    __nv_bfloat16* orow = o + (size_t)(q0 + qr0) * qstride + (size_t)h * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
      *reinterpret_cast<__nv_bfloat162*>(orow + i * 8 + tig * 2) = __floats2bfloat162_rn(acc[i][0] * inv0, acc[i][1] * inv0);
    if (tig == 0) lse[(size_t)h * T + q0 + qr0] = lrow[0] > 0.f ? (mrow[0] + log2f(lrow[0])) * LN2 : -INFINITY;
  }
  if (qr1 < n) {
    __nv_bfloat16* orow = o + (size_t)(q0 + qr1) * qstride + (size_t)h * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
      *reinterpret_cast<__nv_bfloat162*>(orow + i * 8 + tig * 2) = __floats2bfloat162_rn(acc[i][2] * inv1, acc[i][3] * inv1);
    if (tig == 0) lse[(size_t)h * T + q0 + qr1] = lrow[1] > 0.f ? (mrow[1] + log2f(lrow[1])) * LN2 : -INFINITY;
  }
}

// ================================================================================= backward
// delta[h, t] = sum_d dO[t,h,d] * O[t,h,d]
template <int D>
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                  float* __restrict__ delta, int T, int Hq) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const long total = (long)T * Hq;
  for (long it = (long)blockIdx.x * warps + (threadIdx.x >> 5); it < total; it += (long)gridDim.x * warps) {
    const int t = (int)(it / Hq), h = (int)(it % Hq);
    const __nv_bfloat16* a = dout + ((size_t)t * Hq + h) * D;
    const __nv_bfloat16* b = out + ((size_t)t * Hq + h) * D;
    float s = 0.f;
    for (int i = lane; i < D; i += 32) s += __bfloat162float(a[i]) * __bfloat162float(b[i]);
    s = bb::warp_sum(s);
    if (lane == 0) delta[(size_t)h * T + t] = s;
  }
}

// One CTA: 64 keys of one KV head and DH of the D output columns (blockIdx.z = kv head * D/DH + column
// block).  S = QK^T and dP = dO V^T always contract over the full head dim; only the dK / dV / dQ
// columns [c0, c0 + DH) are produced, which keeps the register accumulators of D = 256 at the size
// of the D = 128 case.  mode 0 = own (self) keys of sequence `blockIdx.y`; mode 1 = keys of prefix
// span `blockIdx.y`, read by the sequences users[rowptr[sp]..rowptr[sp+1]).
template <int D, int DH>
__global__ void __launch_bounds__(NWARP * 32, 1) tree_attn_bwd_kernel(
    int mode, const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, const __nv_bfloat16* __restrict__ pk, const __nv_bfloat16* __restrict__ pv,
    const __nv_bfloat16* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ delta,
    const int* __restrict__ cu, const int* __restrict__ users_meta, int nspans, float* __restrict__ dq_acc,
    __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, __nv_bfloat16* __restrict__ dpk,
    __nv_bfloat16* __restrict__ dpv, int T, int Hq, int Hk, float scale, float scale_log2) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int LD = Smem<D>::LD;
  constexpr int LDS = BM + 8;
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sV = sK + BN * LD;
  __nv_bfloat16* sQ = sV + BN * LD;
  __nv_bfloat16* sdO = sQ + BM * LD;
  __nv_bfloat16* sdS = sdO + BM * LD;                         // [BN keys][BM q] (dS^T)
  float* sL = reinterpret_cast<float*>(sdS + BN * LDS);       // lse*log2e per q row
  float* sDl = sL + BM;                                        // delta per q row

  constexpr int NSPLIT = D / DH;
  const int hk = blockIdx.z / NSPLIT;
  const int c0 = (blockIdx.z % NSPLIT) * DH;
  const int rep = Hq / Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const size_t qstride = (size_t)Hq * D, kstride = (size_t)Hk * D;
  const int kb = blockIdx.x * BN;

  // --- which keys / which queries
  int key_len, own_seq = -1, span_off = 0, u_begin = 0, u_end = 0;
  const int* rowptr = users_meta;
  const int* users = users_meta + nspans + 1;
  const int* span_off_a = users + (nspans > 0 ? rowptr[nspans] : 0);
  const int* span_len_a = span_off_a + nspans;
  if (mode == 0) {
    own_seq = blockIdx.y;
    key_len = cu[own_seq + 1] - cu[own_seq];
  } else {
    const int sp = blockIdx.y;
    span_off = span_off_a[sp];
    key_len = span_len_a[sp];
    u_begin = rowptr[sp];
    u_end = rowptr[sp + 1];
  }
  if (kb >= key_len) return;
  const __nv_bfloat16* kbase = (mode == 0) ? k + (size_t)cu[own_seq] * kstride : pk + (size_t)span_off * kstride;
  const __nv_bfloat16* vbase = (mode == 0) ? v + (size_t)cu[own_seq] * kstride : pv + (size_t)span_off * kstride;
  load_tile<D>(sK, [&](int r) -> const __nv_bfloat16* {
    return kb + r < key_len ? kbase + (size_t)(kb + r) * kstride + (size_t)hk * D : nullptr;
  }, k);
  load_tile<D>(sV, [&](int r) -> const __nv_bfloat16* {
    return kb + r < key_len ? vbase + (size_t)(kb + r) * kstride + (size_t)hk * D : nullptr;
  }, v);
  cp_async_commit();

  float dK[DH / 8][4], dV[DH / 8][4];
#pragma unroll
  for (int i = 0; i < DH / 8; ++i) {
    dK[i][0] = dK[i][1] = dK[i][2] = dK[i][3] = 0.f;
    dV[i][0] = dV[i][1] = dV[i][2] = dV[i][3] = 0.f;
  }
  const float LOG2E = 1.4426950408889634f;
  const int nusers = (mode == 0) ? 1 : (u_end - u_begin);
  for (int ui = 0; ui < nusers; ++ui) {
    const int s_idx = (mode == 0) ? own_seq : users[u_begin + ui];
    const int q0 = cu[s_idx], n = cu[s_idx + 1] - q0;
    const int first_tile = (mode == 0) ? kb / BM : 0;  // causal: queries before kb never see these keys
    for (int hh = 0; hh < rep; ++hh) {
      const int h = hk * rep + hh;
      for (int mt = first_tile; mt * BM < n; ++mt) {
        const int m0 = mt * BM;
        __syncthreads();  // previous iteration done with sQ/sdO/sdS
        load_tile<D>(sQ, [&](int r) -> const __nv_bfloat16* {
          return m0 + r < n ? q + (size_t)(q0 + m0 + r) * qstride + (size_t)h * D : nullptr;
        }, q);
        load_tile<D>(sdO, [&](int r) -> const __nv_bfloat16* {
          return m0 + r < n ? dout + (size_t)(q0 + m0 + r) * qstride + (size_t)h * D : nullptr;
        }, dout);
        cp_async_commit();
        for (int r = threadIdx.x; r < BM; r += NWARP * 32) {
          const bool ok = m0 + r < n;
          sL[r] = ok ? lse[(size_t)h * T + q0 + m0 + r] * LOG2E : 0.f;
          sDl[r] = ok ? delta[(size_t)h * T + q0 + m0 + r] : 0.f;
        }
        cp_async_wait<0>();
        __syncthreads();

        // S^T (this warp's 16 keys x 64 q) and dP^T
        float st[8][4], dpt[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
          dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
        }
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          uint32_t ak[4], av[4];
          ldsm_x4(ak[0], ak[1], ak[2], ak[3], sK + (warp * 16 + (lane & 15)) * LD + ks * 16 + (lane >> 4) * 8);
          ldsm_x4(av[0], av[1], av[2], av[3], sV + (warp * 16 + (lane & 15)) * LD + ks * 16 + (lane >> 4) * 8);
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t b0, b1, b2, b3;
            const int roff = (np * 16 + (lane & 7) + (lane >> 4) * 8) * LD + ks * 16 + ((lane >> 3) & 1) * 8;
            ldsm_x4(b0, b1, b2, b3, sQ + roff);
            mma16816(st[2 * np], ak, b0, b1);
            mma16816(st[2 * np + 1], ak, b2, b3);
            ldsm_x4(b0, b1, b2, b3, sdO + roff);
            mma16816(dpt[2 * np], av, b0, b1);
            mma16816(dpt[2 * np + 1], av, b2, b3);
          }
        }
        // P^T, dS^T
        const int key0 = kb + warp * 16 + g, key1 = key0 + 8;  // key index (self local / span local)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int qi = nt * 8 + tig * 2 + (e & 1);  // q row within tile
            const int key = (e < 2) ? key0 : key1;
            bool ok = (m0 + qi < n) && key < key_len && (mode == 1 || key <= m0 + qi);
            float p = ok ? exp2f(st[nt][e] * scale_log2 - sL[qi]) : 0.f;
            st[nt][e] = p;
            dpt[nt][e] = p * (dpt[nt][e] - sDl[qi]);
          }
        }
        // write dS^T (bf16) for the dQ GEMM
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          *reinterpret_cast<uint32_t*>(sdS + (warp * 16 + g) * LDS + nt * 8 + tig * 2) = pack_bf16(dpt[nt][0], dpt[nt][1]);
          *reinterpret_cast<uint32_t*>(sdS + (warp * 16 + g + 8) * LDS + nt * 8 + tig * 2) =
              pack_bf16(dpt[nt][2], dpt[nt][3]);
        }
        // dV += P^T dO ; dK += dS^T Q   (k dim = 64 q rows -> 4 k-steps)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t ap[4], ad[4];
          ap[0] = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
          ap[1] = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
          ap[2] = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
          ap[3] = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
          ad[0] = pack_bf16(dpt[2 * kk][0], dpt[2 * kk][1]);
          ad[1] = pack_bf16(dpt[2 * kk][2], dpt[2 * kk][3]);
          ad[2] = pack_bf16(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
          ad[3] = pack_bf16(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
          for (int dp = 0; dp < DH / 16; ++dp) {
            uint32_t b0, b1, b2, b3;
            const int off = (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + c0 + dp * 16 + (lane >> 4) * 8;
            ldsm_x4_t(b0, b1, b2, b3, sdO + off);
            mma16816(dV[2 * dp], ap, b0, b1);
            mma16816(dV[2 * dp + 1], ap, b2, b3);
            ldsm_x4_t(b0, b1, b2, b3, sQ + off);
            mma16816(dK[2 * dp], ad, b0, b1);
            mma16816(dK[2 * dp + 1], ad, b2, b3);
          }
        }
        __syncthreads();
        // dQ (this warp's 16 q rows x D) = dS K over the 64 keys
        {
          float dq[DH / 8][4];
#pragma unroll
          for (int i = 0; i < DH / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            uint32_t a[4];
            // A[q][key] from dS^T[key][q] via transposed ldmatrix
            ldsm_x4_t(a[0], a[1], a[2], a[3],
                      sdS + (kk * 16 + (lane & 7) + (lane >> 4) * 8) * LDS + warp * 16 + ((lane >> 3) & 1) * 8);
#pragma unroll
            for (int dp = 0; dp < DH / 16; ++dp) {
              uint32_t b0, b1, b2, b3;
              ldsm_x4_t(b0, b1, b2, b3,
                        sK + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + c0 + dp * 16 + (lane >> 4) * 8);
              mma16816(dq[2 * dp], a, b0, b1);
              mma16816(dq[2 * dp + 1], a, b2, b3);
            }
          }
          const int r0 = m0 + warp * 16 + g, r1 = r0 + 8;
#pragma unroll
          for (int i = 0; i < DH / 8; ++i) {
            const int col = c0 + i * 8 + tig * 2;
            if (r0 < n) {
              float* dst = dq_acc + (size_t)(q0 + r0) * qstride + (size_t)h * D + col;
              atomicAdd(dst, dq[i][0] * scale);
              atomicAdd(dst + 1, dq[i][1] * scale);
            }
            if (r1 < n) {
              float* dst = dq_acc + (size_t)(q0 + r1) * qstride + (size_t)h * D + col;
              atomicAdd(dst, dq[i][2] * scale);
              atomicAdd(dst + 1, dq[i][3] * scale);
            }
          }
        }
      }
    }
  }
  // write dK (scaled) and dV for this warp's 16 keys
  __nv_bfloat16* dkb = (mode == 0) ? dk + (size_t)cu[own_seq] * kstride : dpk + (size_t)span_off * kstride;
  __nv_bfloat16* dvb = (mode == 0) ? dv + (size_t)cu[own_seq] * kstride : dpv + (size_t)span_off * kstride;
  const int key0 = kb + warp * 16 + g, key1 = key0 + 8;
#pragma unroll
  for (int i = 0; i < DH / 8; ++i) {
    const int col = c0 + i * 8 + tig * 2;
    if (key0 < key_len) {
      *reinterpret_cast<__nv_bfloat162*>(dkb + (size_t)key0 * kstride + (size_t)hk * D + col) =
          __floats2bfloat162_rn(dK[i][0] * scale, dK[i][1] * scale);
      *reinterpret_cast<__nv_bfloat162*>(dvb + (size_t)key0 * kstride + (size_t)hk * D + col) =
          __floats2bfloat162_rn(dV[i][0], dV[i][1]);
    }
    if (key1 < key_len) {
      *reinterpret_cast<__nv_bfloat162*>(dkb + (size_t)key1 * kstride + (size_t)hk * D + col) =
          __floats2bfloat162_rn(dK[i][2] * scale, dK[i][3] * scale);
      *reinterpret_cast<__nv_bfloat162*>(dvb + (size_t)key1 * kstride + (size_t)hk * D + col) =
          __floats2bfloat162_rn(dV[i][2], dV[i][3]);
    }
  }
}

template <int D>
size_t fwd_smem() {
  return (size_t)(BM + 4 * BN) * Smem<D>::LD * sizeof(__nv_bfloat16);
}
template <int D>
size_t bwd_smem() {
  return (size_t)(2 * BN + 2 * BM) * Smem<D>::LD * sizeof(__nv_bfloat16) + (size_t)BN * (BM + 8) * 2 +
         2 * BM * sizeof(float);
}

}  // namespace

std::vector<torch::Tensor> tree_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor pk,
                                         torch::Tensor pv, torch::Tensor cu, torch::Tensor poff, torch::Tensor plen,
                                         int64_t max_seqlen, int64_t max_prefix, double scale) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16, "q must be CUDA bf16");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "q/k/v must be contiguous");
  const int T = q.size(0), Hq = q.size(1), D = q.size(2), Hk = k.size(1);
  TORCH_CHECK(Hq % Hk == 0, "GQA: Hq % Hkv");
  TORCH_CHECK(cu.scalar_type() == at::kInt && poff.scalar_type() == at::kInt && plen.scalar_type() == at::kInt,
              "metadata must be int32");
  const int B = cu.numel() - 1;
  auto o = torch::empty_like(q);
  auto lse = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  if (T == 0 || B == 0) return {o, lse};
  const __nv_bfloat16* pkp = pk.numel() ? (const __nv_bfloat16*)pk.data_ptr() : (const __nv_bfloat16*)k.data_ptr();
  const __nv_bfloat16* pvp = pv.numel() ? (const __nv_bfloat16*)pv.data_ptr() : (const __nv_bfloat16*)v.data_ptr();
  dim3 grid((max_seqlen + BM - 1) / BM, B, Hq);
  const float sl2 = (float)(scale * 1.4426950408889634);
  auto stream = at::cuda::getCurrentCUDAStream();
#define BB_FWD(DD)                                                                                             \
  {                                                                                                            \
    auto kern = tree_attn_fwd_kernel<DD>;                                                                      \
    size_t sm = fwd_smem<DD>();                                                                                \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                          \
    kern<<<grid, NWARP * 32, sm, stream>>>((const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), \
                                           (const __nv_bfloat16*)v.data_ptr(), pkp, pvp, cu.data_ptr<int>(),       \
                                           poff.data_ptr<int>(), plen.data_ptr<int>(), (__nv_bfloat16*)o.data_ptr(), \
                                           lse.data_ptr<float>(), T, Hq, Hk, sl2);                              \
  }
  if (D == 128) {
    BB_FWD(128)
  } else if (D == 64) {
    BB_FWD(64)
  } else if (D == 256) {
    BB_FWD(256)
  } else {
    TORCH_CHECK(false, "tree attention: head_dim must be 64, 128 or 256");
  }
#undef BB_FWD
  BB_POST_LAUNCH();
  return {o, lse};
}

std::vector<torch::Tensor> tree_attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                         torch::Tensor pk, torch::Tensor pv, torch::Tensor o, torch::Tensor lse,
                                         torch::Tensor cu, torch::Tensor poff, torch::Tensor plen, int64_t max_seqlen,
                                         int64_t max_prefix, double scale, torch::Tensor users_meta,
                                         int64_t nspans_in) {
  const int T = q.size(0), Hq = q.size(1), D = q.size(2), Hk = k.size(1);
  const int B = cu.numel() - 1;
  auto dq_acc = torch::zeros({T, Hq, D}, q.options().dtype(at::kFloat));
  auto dk = torch::empty_like(k), dv = torch::empty_like(v);
  auto dpk = torch::zeros_like(pk), dpv = torch::zeros_like(pv);
  auto delta = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  if (T == 0 || B == 0) return {dq_acc.to(at::kBFloat16), dk, dv, dpk, dpv};
  auto stream = at::cuda::getCurrentCUDAStream();
  // users_meta: [rowptr(nspans+1) | users | span_off | span_len | nspans]  (nspans also passed from the host)
  const int nspans = (int)nspans_in;
  const float sl2 = (float)(scale * 1.4426950408889634);
  const __nv_bfloat16* pkp = pk.numel() ? (const __nv_bfloat16*)pk.data_ptr() : (const __nv_bfloat16*)k.data_ptr();
  const __nv_bfloat16* pvp = pv.numel() ? (const __nv_bfloat16*)pv.data_ptr() : (const __nv_bfloat16*)v.data_ptr();
  __nv_bfloat16* dpkp = dpk.numel() ? (__nv_bfloat16*)dpk.data_ptr() : nullptr;
  __nv_bfloat16* dpvp = dpv.numel() ? (__nv_bfloat16*)dpv.data_ptr() : nullptr;
#define BB_BWD(DD, DHH)                                                                                            \
  {                                                                                                                \
    attn_delta_kernel<DD><<<std::max(1, std::min((T * Hq + 7) / 8, 148 * 8)), 256, 0, stream>>>(                  \
        (const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)o.data_ptr(), delta.data_ptr<float>(), T, Hq); \
    bb::launch_counter().fetch_add(nspans > 0 && max_prefix > 0 ? 3 : 2);                                          \
    auto kern = tree_attn_bwd_kernel<DD, DHH>;                                                                     \
    size_t sm = bwd_smem<DD>();                                                                                    \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                              \
    dim3 g0((max_seqlen + BN - 1) / BN, B, Hk * (DD / DHH));                                                       \
    kern<<<g0, NWARP * 32, sm, stream>>>(0, (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), \
                                         (const __nv_bfloat16*)v.data_ptr(), pkp, pvp,                             \
                                         (const __nv_bfloat16*)dout.data_ptr(), lse.data_ptr<float>(),             \
                                         delta.data_ptr<float>(), cu.data_ptr<int>(), users_meta.data_ptr<int>(),  \
                                         nspans, dq_acc.data_ptr<float>(), (__nv_bfloat16*)dk.data_ptr(),          \
                                         (__nv_bfloat16*)dv.data_ptr(), dpkp, dpvp, T, Hq, Hk, (float)scale, sl2); \
    if (nspans > 0 && max_prefix > 0) {                                                                            \
      dim3 g1((max_prefix + BN - 1) / BN, nspans, Hk * (DD / DHH));                                                \
      kern<<<g1, NWARP * 32, sm, stream>>>(1, (const __nv_bfloat16*)q.data_ptr(),                                 \
                                           (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(), \
                                           pkp, pvp, (const __nv_bfloat16*)dout.data_ptr(), lse.data_ptr<float>(), \
                                           delta.data_ptr<float>(), cu.data_ptr<int>(),                            \
                                           users_meta.data_ptr<int>(), nspans, dq_acc.data_ptr<float>(),           \
                                           (__nv_bfloat16*)dk.data_ptr(), (__nv_bfloat16*)dv.data_ptr(), dpkp,     \
                                           dpvp, T, Hq, Hk, (float)scale, sl2);                                    \
    }                                                                                                              \
  }
  if (D == 128) {
    BB_BWD(128, 128)
  } else if (D == 64) {
    BB_BWD(64, 64)
  } else if (D == 256) {
    BB_BWD(256, 128)
  } else {
    TORCH_CHECK(false, "tree attention backward: head_dim must be 64, 128 or 256");
  }
#undef BB_BWD
  BB_CHECK_CUDA(cudaGetLastError());
  return {dq_acc.to(at::kBFloat16), dk, dv, dpk, dpv};
}
