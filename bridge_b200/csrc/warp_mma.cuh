// Warp-level bf16 tensor-core tiles (mma.sync m16n8k16, FP32 accumulate) over shared-memory operands.
//
// warp_tile<A_T, B_KMAJ>(c, A, lda, B, ldb, m0, n0, K) accumulates the 16 x 16 block
//   C[m0:m0+16, n0:n0+16] += A[m0:m0+16, 0:K] * B[0:K, n0:n0+16]
// where A is stored row-major [M][K] (A_T = false) or as its transpose [K][M] (A_T = true), and B is
// stored [N][K] (B_KMAJ = true) or [K][N] (B_KMAJ = false).  Leading dimensions are in elements and
// must keep every 8-element row segment 16-byte aligned.  Fragment c[j][e] holds row
//   m0 + (lane >> 2) + 8 * (e >> 1), column n0 + 8 * j + 2 * (lane & 3) + (e & 1).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace wm {

__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr(p)));
}
__device__ __forceinline__ void ldsm4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr(p)));
}
__device__ __forceinline__ void mma(float* c, const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool A_T, bool B_KMAJ>
__device__ __forceinline__ void warp_tile(float (&c)[2][4], const __nv_bfloat16* A, int lda, const __nv_bfloat16* B,
                                          int ldb, int m0, int n0, int K) {
  const int lane = threadIdx.x & 31;
#pragma unroll 4
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t a[4], b[4];
    if (A_T) ldsm4_t(a, A + (size_t)(k0 + (lane & 7) + (lane >> 4) * 8) * lda + m0 + ((lane >> 3) & 1) * 8);
    else ldsm4(a, A + (size_t)(m0 + (lane & 15)) * lda + k0 + (lane >> 4) * 8);
    if (B_KMAJ) ldsm4(b, B + (size_t)(n0 + (lane & 7) + (lane >> 4) * 8) * ldb + k0 + ((lane >> 3) & 1) * 8);
    else ldsm4_t(b, B + (size_t)(k0 + (lane & 7) + ((lane >> 3) & 1) * 8) * ldb + n0 + (lane >> 4) * 8);
    mma(c[0], a, b[0], b[1]);
    mma(c[1], a, b[2], b[3]);
  }
}

// C[M, N] = A * B over all warps of the block; `epi(row, col, value)` receives every element.
template <bool A_T, bool B_KMAJ, typename Epi>
__device__ __forceinline__ void block_gemm(int M, int N, int K, const __nv_bfloat16* A, int lda,
                                           const __nv_bfloat16* B, int ldb, Epi epi) {
  const int warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int tn = N / 16, tiles = (M / 16) * tn;
  for (int t = warp; t < tiles; t += nwarp) {
    const int m0 = (t / tn) * 16, n0 = (t % tn) * 16;
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    warp_tile<A_T, B_KMAJ>(c, A, lda, B, ldb, m0, n0, K);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        epi(m0 + (lane >> 2) + 8 * (e >> 1), n0 + 8 * j + 2 * (lane & 3) + (e & 1), c[j][e]);
  }
}

}  // namespace wm

namespace wm {

// As block_gemm, with B given as an unevaluated bf16 sum Bhi + Blo (an FP32 matrix split into its bf16
// rounding and the bf16 rounding of the remainder): two tensor-core passes, ~16 significant bits of B.
template <bool A_T, bool B_KMAJ, typename Epi>
__device__ __forceinline__ void block_gemm2(int M, int N, int K, const __nv_bfloat16* A, int lda,
                                            const __nv_bfloat16* Bhi, const __nv_bfloat16* Blo, int ldb, Epi epi) {
  const int warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int tn = N / 16, tiles = (M / 16) * tn;
  for (int t = warp; t < tiles; t += nwarp) {
    const int m0 = (t / tn) * 16, n0 = (t % tn) * 16;
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    warp_tile<A_T, B_KMAJ>(c, A, lda, Bhi, ldb, m0, n0, K);
    warp_tile<A_T, B_KMAJ>(c, A, lda, Blo, ldb, m0, n0, K);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        epi(m0 + (lane >> 2) + 8 * (e >> 1), n0 + 8 * j + 2 * (lane & 3) + (e & 1), c[j][e]);
  }
}

// hi / lo bf16 split of an FP32 value
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16(x);
  lo = __float2bfloat16(x - __bfloat162float(hi));
}

}  // namespace wm

namespace wm {

// As block_gemm (or block_gemm2 when Blo != nullptr), for epilogues that also sum per-row and per-column
// contributions into shared-memory vectors: `epi(row, col, value, rc, cc)` adds to rc[0..1] (summed
// into rdst0[row], rdst1[row]) and cc[0] (summed into cdst[col]).  The sums are reduced inside each
// warp's 16 x 16 tile with shuffles first, so a tile issues 16 shared atomics per vector instead of one
// per element (the per-element form serialises on the four lanes that share a row).  Null destinations
// are skipped.
template <bool A_T, bool B_KMAJ, typename Epi>
__device__ __forceinline__ void block_gemm_red(int M, int N, int K, const __nv_bfloat16* A, int lda,
                                               const __nv_bfloat16* B, const __nv_bfloat16* Blo, int ldb,
                                               float* rdst0, float* rdst1, float* cdst, Epi epi) {
  const int warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int tn = N / 16, tiles = (M / 16) * tn;
  for (int t = warp; t < tiles; t += nwarp) {
    const int m0 = (t / tn) * 16, n0 = (t % tn) * 16;
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    warp_tile<A_T, B_KMAJ>(c, A, lda, B, ldb, m0, n0, K);
    if (Blo != nullptr) warp_tile<A_T, B_KMAJ>(c, A, lda, Blo, ldb, m0, n0, K);
    float racc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};   // [row half][vector]
    float cacc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};   // [j][e & 1]
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float rc[2] = {0.f, 0.f}, cc[1] = {0.f};
        epi(m0 + (lane >> 2) + 8 * (e >> 1), n0 + 8 * j + 2 * (lane & 3) + (e & 1), c[j][e], rc, cc);
        racc[e >> 1][0] += rc[0];
        racc[e >> 1][1] += rc[1];
        cacc[j][e & 1] += cc[0];
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v = racc[hh][k];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        float* dst = k == 0 ? rdst0 : rdst1;
        if (dst != nullptr && (lane & 3) == 0 && v != 0.f) atomicAdd(&dst[m0 + (lane >> 2) + 8 * hh], v);
      }
    if (cdst != nullptr) {
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          float v = cacc[j][b];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          if (lane < 4 && v != 0.f) atomicAdd(&cdst[n0 + 8 * j + 2 * lane + b], v);
        }
    }
  }
}

}  // namespace wm

namespace wm {

// As block_gemm / block_gemm2 (Blo != nullptr), with the epilogue called once per pair of adjacent
// columns: `epi(row, col, value(col), value(col + 1))`, col even (vector stores / float2 atomics).
template <bool A_T, bool B_KMAJ, typename Epi>
__device__ __forceinline__ void block_gemm_pairs(int M, int N, int K, const __nv_bfloat16* A, int lda,
                                                 const __nv_bfloat16* B, const __nv_bfloat16* Blo, int ldb, Epi epi) {
  const int warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int tn = N / 16, tiles = (M / 16) * tn;
  for (int t = warp; t < tiles; t += nwarp) {
    const int m0 = (t / tn) * 16, n0 = (t % tn) * 16;
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    warp_tile<A_T, B_KMAJ>(c, A, lda, B, ldb, m0, n0, K);
    if (Blo != nullptr) warp_tile<A_T, B_KMAJ>(c, A, lda, Blo, ldb, m0, n0, K);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2)
        epi(m0 + (lane >> 2) + 8 * (e >> 1), n0 + 8 * j + 2 * (lane & 3), c[j][e], c[j][e + 1]);
  }
}

}  // namespace wm
