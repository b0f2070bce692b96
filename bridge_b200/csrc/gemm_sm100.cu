// Persistent tcgen05 GEMM for sm_100a:  C[M,N] (+)= A[M,K] * B[N,K]^T, bf16 operands, FP32 accumulate.
//
// * A and B may each be K-major (row-major [rows, K]) or MN-major (the transposed operand stored
//   row-major as [K, rows]) -- so a linear layer's forward (x W^T), data gradient (dy W) and
//   weight gradient (dy^T x) all run without a transpose copy.
// * Tiles 128 x 256 x 64, 4-stage TMA ring (128-byte swizzle), accumulators double-buffered in
//   TMEM (2 x 256 columns) so the epilogue of tile i overlaps the main loop of tile i+1.
// * Warp roles (192 threads): warp 0 issues TMA, warp 1 owns TMEM and issues tcgen05.mma (one
//   thread), warps 2-5 drain TMEM (tcgen05.ld) and write C -- bf16 store, or FP32
//   read-add-write (used to accumulate weight gradients straight into the FP32 main-grad arena).
// * One CTA per SM, tiles swizzled in groups of 8 M-tiles for L2 reuse.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "sm100_common.cuh"

static bool gemm_trace() {
  static int v = -1;
  if (v < 0) v = getenv("BB_GEMM_TRACE") ? 1 : 0;
  return v == 1;
}
#define GTRACE(msg) \
  do {              \
    if (gemm_trace()) { fprintf(stderr, "[gemm] %s\n", msg); fflush(stderr); } \
  } while (0)


namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;

struct SmemLayout {
  // stage buffers come first (1024-byte aligned by construction)
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = STAGES * A_BYTES;
  static constexpr int BAR_OFF = B_OFF + STAGES * B_BYTES;
  static constexpr int EPI_OFF = BAR_OFF + 256;              // RS epilogue staging: 4 warps x 32 x 33 words
  static constexpr int TOTAL = BAR_OFF + 256;
  static constexpr int TOTAL_EPI = EPI_OFF + 4 * 32 * 33 * 4;
};

template <bool A_MN, bool B_MN, bool ACCUM_F32>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, void* C,
                int M, int N, int K, long ldc, int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // Align the dynamic buffer to 1024 B (128-byte swizzle atoms).
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem + SmemLayout::A_OFF;
  unsigned char* sB = smem + SmemLayout::B_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int nk = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tfull[a], 1);
      sm100::mbar_init(&tempty[a], 128);
    }
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tmap_a);
    sm100::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, TMEM_COLS);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto tile_coords = [&](int t, int& m0, int& n0) {
    // group-of-8 M raster for L2 reuse of B tiles
    const int group = 8;
    const int per_group = group * n_tiles;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gm = min(group, m_tiles - first_m);
    const int r = t % per_group;
    m0 = (first_m + r % gm) * BM;
    n0 = (r / gm) * BN;
  };

  constexpr uint32_t IDESC = sm100::umma_idesc_bf16(BM, BN, A_MN, B_MN);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int m0, n0;
        tile_coords(t, m0, n0);
        for (int kb = 0; kb < nk; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1, err, 1)) {
            ok = false;
            break;
          }
          sm100::mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          unsigned char* a_dst = sA + stage * A_BYTES;
          unsigned char* b_dst = sB + stage * B_BYTES;
          if (A_MN) {
#pragma unroll
            for (int i = 0; i < BM / 64; ++i)
              sm100::tma_load_2d(a_dst + i * 8192, &tmap_a, &full[stage], m0 + 64 * i, kb * BK);
          } else {
            sm100::tma_load_2d(a_dst, &tmap_a, &full[stage], kb * BK, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              sm100::tma_load_2d(b_dst + i * 8192, &tmap_b, &full[stage], n0 + 64 * i, kb * BK);
          } else {
            sm100::tma_load_2d(b_dst, &tmap_b, &full[stage], kb * BK, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!sm100::mbar_wait(&tempty[acc], acc_phase ^ 1, err, 2)) break;
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!sm100::mbar_wait(&full[stage], phase, err, 3)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_addr(sA + stage * A_BYTES);
          const uint32_t b_base = sm100::smem_addr(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sm100::umma_desc_sw128(a_base + kk * 2048, 8192, 1024)
                                     : sm100::umma_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sm100::umma_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                     : sm100::umma_desc_sw128(b_base + kk * 32, 16, 1024);
            sm100::umma_bf16(d_tmem, ad, bd, IDESC, (kb | kk) != 0);
          }
          sm100::umma_commit(&empty[stage]);  // stage reusable once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        sm100::umma_commit(&tfull[acc]);      // accumulator complete
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int m0, n0;
      tile_coords(t, m0, n0);
      const bool got = sm100::mbar_wait(&tfull[acc], acc_phase, err, 4);
      if (!__all_sync(0xffffffffu, got)) break;  // keep the warp converged for tcgen05.ld
      sm100::tc_fence_after();
      const int row = m0 + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(t_row + c * 32, r);
        sm100::tmem_ld_wait();
        const int col0 = n0 + c * 32;
        if (row < M && col0 < N) {
          if (ACCUM_F32) {
            float* dst = reinterpret_cast<float*>(C) + (size_t)row * ldc + col0;
            if (col0 + 32 <= N) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                float4 v = reinterpret_cast<float4*>(dst)[j];
                v.x += __uint_as_float(r[4 * j]);
                v.y += __uint_as_float(r[4 * j + 1]);
                v.z += __uint_as_float(r[4 * j + 2]);
                v.w += __uint_as_float(r[4 * j + 3]);
                reinterpret_cast<float4*>(dst)[j] = v;
              }
            } else {
              for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] += __uint_as_float(r[j]);
            }
          } else {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (size_t)row * ldc + col0;
            if (col0 + 32 <= N) {
              uint32_t p[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                p[j] = *reinterpret_cast<uint32_t*>(&h);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(dst)[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
            } else {
              for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] = __float2bfloat16(__uint_as_float(r[j]));
            }
          }
        }
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2): a cluster of two CTAs on two SMs computes a 256 x 256 tile.
// CTA r stages rows [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the B tile
// (N half) -- 32 KB per stage instead of 48 KB, so 6 stages fit and every B row is fetched once per
// pair.  The leader (rank 0) issues the M = 256 MMAs; both CTAs' TMA loads complete on the leader's
// `full` barrier; the MMA commits arrive on both CTAs' `empty` / `tfull` barriers (multicast commit);
// both CTAs' epilogue threads arrive on the leader's `tempty`.  Each CTA drains its own TMEM rows.
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2;  // 16 KB
constexpr int P_B_BYTES = 128 * BK * 2;  // 16 KB (this CTA's half of the 256-row B tile)

struct PairSmem {
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = P_STAGES * P_A_BYTES;
  static constexpr int BAR_OFF = B_OFF + P_STAGES * P_B_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256;
};

template <bool A_MN, bool B_MN, bool ACCUM_F32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, void* C,
                     int M, int N, int K, long ldc, int* err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem + PairSmem::A_OFF;
  unsigned char* sB = smem + PairSmem::B_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PairSmem::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + P_STAGES;
  uint64_t* tfull = bars + 2 * P_STAGES;
  uint64_t* tempty = bars + 2 * P_STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (M + 255) / 256, n_tiles = (N + 255) / 256;
  const int num_tiles = m_tiles * n_tiles;
  const int nk = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tfull[a], 1);
      sm100::mbar_init(&tempty[a], 256);
    }
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tmap_a);
    sm100::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) sm100::tmem_alloc_pair(tmem_slot, TMEM_COLS);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // both CTAs' barriers are initialised before any remote arrive / TMA
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto tile_coords = [&](int t, int& m0, int& n0) {
    const int group = 8;
    const int per_group = group * n_tiles;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gm = min(group, m_tiles - first_m);
    const int r = t % per_group;
    m0 = (first_m + r % gm) * 256;
    n0 = (r / gm) * 256;
  };

  constexpr uint32_t IDESC = sm100::umma_idesc_bf16(256, 256, A_MN, B_MN);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        int m0, n0;
        tile_coords(t, m0, n0);
        const int ma = m0 + 128 * (int)rank, nb = n0 + 128 * (int)rank;
        for (int kb = 0; kb < nk; ++kb) {
          if (!sm100::mbar_wait_cluster(&empty[stage], phase ^ 1, err, 11)) {
            ok = false;
            break;
          }
          if (leader) sm100::mbar_expect_tx(&full[stage], 2 * (P_A_BYTES + P_B_BYTES));
          const uint32_t fb = sm100::mapa(sm100::smem_addr(&full[stage]), 0);
          unsigned char* a_dst = sA + stage * P_A_BYTES;
          unsigned char* b_dst = sB + stage * P_B_BYTES;
          if (A_MN) {
            sm100::tma_load_2d_pair(a_dst, &tmap_a, fb, ma, kb * BK);
            sm100::tma_load_2d_pair(a_dst + 8192, &tmap_a, fb, ma + 64, kb * BK);
          } else {
            sm100::tma_load_2d_pair(a_dst, &tmap_a, fb, kb * BK, ma);
          }
          if (B_MN) {
            sm100::tma_load_2d_pair(b_dst, &tmap_b, fb, nb, kb * BK);
            sm100::tma_load_2d_pair(b_dst + 8192, &tmap_b, fb, nb + 64, kb * BK);
          } else {
            sm100::tma_load_2d_pair(b_dst, &tmap_b, fb, kb * BK, nb);
          }
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        if (!sm100::mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, err, 12)) break;
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        for (int kb = 0; kb < nk; ++kb) {
          if (!sm100::mbar_wait_cluster(&full[stage], phase, err, 13)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_addr(sA + stage * P_A_BYTES);
          const uint32_t b_base = sm100::smem_addr(sB + stage * P_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sm100::umma_desc_sw128(a_base + kk * 2048, 8192, 1024)
                                     : sm100::umma_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sm100::umma_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                     : sm100::umma_desc_sw128(b_base + kk * 32, 16, 1024);
            sm100::umma_bf16_pair(d_tmem, ad, bd, IDESC, (kb | kk) != 0);
          }
          sm100::umma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        sm100::umma_commit_pair_mc(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < num_tiles; t += npairs) {
      int m0, n0;
      tile_coords(t, m0, n0);
      const bool got = sm100::mbar_wait_cluster(&tfull[acc], acc_phase, err, 14);
      if (!__all_sync(0xffffffffu, got)) break;
      sm100::tc_fence_after();
      const int row = m0 + 128 * (int)rank + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * 256;
#pragma unroll 1
      for (int c = 0; c < 256 / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(t_row + c * 32, r);
        sm100::tmem_ld_wait();
        const int col0 = n0 + c * 32;
        if (row < M && col0 < N) {
          if (ACCUM_F32) {
            float* dst = reinterpret_cast<float*>(C) + (size_t)row * ldc + col0;
            if (col0 + 32 <= N) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                float4 v = reinterpret_cast<float4*>(dst)[j];
                v.x += __uint_as_float(r[4 * j]);
                v.y += __uint_as_float(r[4 * j + 1]);
                v.z += __uint_as_float(r[4 * j + 2]);
                v.w += __uint_as_float(r[4 * j + 3]);
                reinterpret_cast<float4*>(dst)[j] = v;
              }
            } else {
              for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] += __uint_as_float(r[j]);
            }
          } else {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (size_t)row * ldc + col0;
            if (col0 + 32 <= N) {
              uint32_t p[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                p[j] = *reinterpret_cast<uint32_t*>(&h);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(dst)[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
            } else {
              for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] = __float2bfloat16(__uint_as_float(r[j]));
            }
          }
        }
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive_cluster(sm100::mapa(sm100::smem_addr(&tempty[acc]), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // the peer's smem / barriers stay alive until both CTAs are done
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    BB_CHECK_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [rows, cols] (cols contiguous), box {64, box_rows}.
// Written in place: CUtensorMap is a 64-byte-aligned type and is never copied through the stack.
void make_map(CUtensorMap* m, const void* base, long rows, long cols, long ld, int box_rows) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(m) & 63) == 0, "tensor map storage must be 64-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
}

// Per-thread, explicitly aligned storage for the two maps of one launch.
struct alignas(64) MapPair {
  CUtensorMap a, b;
};
MapPair* map_storage() {
  thread_local MapPair* p = nullptr;
  if (!p) {
    void* raw = nullptr;
    TORCH_CHECK(posix_memalign(&raw, 64, sizeof(MapPair)) == 0, "posix_memalign failed");
    p = reinterpret_cast<MapPair*>(raw);
  }
  return p;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int d;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
  }
  return n;
}

torch::Tensor& error_word() {
  static torch::Tensor e;
  if (!e.defined()) e = torch::zeros({1}, torch::dtype(torch::kInt).device(torch::kCUDA));
  return e;
}

template <bool A_MN, bool B_MN, bool ACC>
void launch(const MapPair* maps, void* c, int M, int N, int K, long ldc) {
  auto kern = gemm_kernel<A_MN, B_MN, ACC>;
  const int smem = SmemLayout::TOTAL + 1024;
  static unsigned long long attr_done = 0;
  bb::set_smem_attr_once(kern, smem, attr_done);
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, num_sms()));
  GTRACE("launch: attr ok");
  int* err = error_word().data_ptr<int>();
  GTRACE("launch: err word");
  // Arguments are passed by address: the runtime copies each by its declared size.
  void* args[] = {const_cast<CUtensorMap*>(&maps->a), const_cast<CUtensorMap*>(&maps->b), &c, &M, &N, &K, &ldc, &err};
  BB_CHECK_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(NUM_THREADS), args, smem,
                                 at::cuda::getCurrentCUDAStream()));
  GTRACE("launched");
  BB_POST_LAUNCH();
}

template <bool A_MN, bool B_MN, bool ACC>
void launch_pair(const MapPair* maps, void* c, int M, int N, int K, long ldc) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, ACC>;
  const int smem = PairSmem::TOTAL + 1024;
  static unsigned long long attr_done = 0;
  bb::set_smem_attr_once(kern, smem, attr_done);
  const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
  const int grid = 2 * std::max(1, std::min(tiles, num_sms() / 2));
  int* err = error_word().data_ptr<int>();
  void* args[] = {const_cast<CUtensorMap*>(&maps->a), const_cast<CUtensorMap*>(&maps->b), &c, &M, &N, &K, &ldc, &err};
  BB_CHECK_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(NUM_THREADS), args, smem,
                                 at::cuda::getCurrentCUDAStream()));
  BB_POST_LAUNCH();
}

bool use_pair(long M, long N) {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("BB_GEMM_PAIR");
    mode = (e && e[0] == '0') ? 0 : 1;
  }
  return mode == 1 && M >= 256 && N >= 256;
}

}  // namespace

// C = op(A) * op(B)^T where op(A) is [M, K] and op(B) is [N, K].
//   a_mn=false: A given as [M, K] (K contiguous);  a_mn=true: A given as [K, M] (M contiguous).
//   b_mn=false: B given as [N, K];                 b_mn=true: B given as [K, N].
// out: bf16 [M, N] written, or fp32 [M, N] accumulated into when `accumulate`.
torch::Tensor gemm(torch::Tensor a, torch::Tensor b, bool a_mn, bool b_mn, c10::optional<torch::Tensor> out,
                   bool accumulate) {
  GTRACE("enter");
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "gemm operands must be CUDA bf16");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "gemm operands: 2-D row-major");
  const long M = a_mn ? a.size(1) : a.size(0);
  const long K = a_mn ? a.size(0) : a.size(1);
  const long N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm: inner dimensions differ");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "gemm: operand row strides must be multiples of 8");
  torch::Tensor c;
  if (out.has_value()) {
    c = *out;
    TORCH_CHECK(c.size(0) == M && c.size(1) == N && c.stride(1) == 1 && c.stride(0) % 8 == 0, "gemm: bad out shape");
    TORCH_CHECK(accumulate ? c.scalar_type() == at::kFloat : c.scalar_type() == at::kBFloat16, "gemm: out dtype");
  } else {
    TORCH_CHECK(!accumulate, "accumulate needs an out tensor");
    c = torch::empty({M, N}, a.options());
  }
  if (M == 0 || N == 0) return c;
  if (K == 0) {
    if (!accumulate) c.zero_();
    return c;
  }
  GTRACE("out ready");
  // The tensor-map encoder needs a current context in the calling thread; autograd worker threads
  // and fresh Python threads may not have made any runtime call yet.
  at::cuda::CUDAGuard device_guard(a.get_device());
  {
    CUcontext cur = nullptr;
    if (cuCtxGetCurrent(&cur) != CUDA_SUCCESS || cur == nullptr) BB_CHECK_CUDA(cudaFree(nullptr));
  }
  MapPair* maps = map_storage();
  GTRACE("storage");
  const bool pair = use_pair(M, N);
  if (a_mn) make_map(&maps->a, a.data_ptr(), K, M, a.stride(0), 64);
  else make_map(&maps->a, a.data_ptr(), M, K, a.stride(0), BM);
  if (b_mn) make_map(&maps->b, b.data_ptr(), K, N, b.stride(0), 64);
  else make_map(&maps->b, b.data_ptr(), N, K, b.stride(0), pair ? 128 : BN);
  GTRACE("maps encoded");
  const long ldc = c.stride(0);
#define BB_G(AM, BMN, ACC)                                                           \
  do {                                                                               \
    if (pair) launch_pair<AM, BMN, ACC>(maps, c.data_ptr(), (int)M, (int)N, (int)K, ldc); \
    else launch<AM, BMN, ACC>(maps, c.data_ptr(), (int)M, (int)N, (int)K, ldc);      \
  } while (0)
  if (accumulate) {
    if (!a_mn && !b_mn) BB_G(false, false, true);
    else if (!a_mn && b_mn) BB_G(false, true, true);
    else if (a_mn && !b_mn) BB_G(true, false, true);
    else BB_G(true, true, true);
  } else {
    if (!a_mn && !b_mn) BB_G(false, false, false);
    else if (!a_mn && b_mn) BB_G(false, true, false);
    else if (a_mn && !b_mn) BB_G(true, false, false);
    else BB_G(true, true, false);
  }
#undef BB_G
  return c;
}

int64_t gemm_error_code() { return error_word().item<int>(); }

// ================================================================================================
// Tensor-parallel GEMMs fused with their collective over NVLink peer memory (sequence parallel).
//
//   AG mode  C[M, N] = A_full[M, K] B^T, where rank j holds rows [j*Ms, (j+1)*Ms) of A in its
//            symmetric staging buffer.  At kernel start the four epilogue warps of every CTA pull
//            the peers' rows into the local A_full buffer (16-byte P2P loads, each remote row crosses
//            NVLink once) and bump a per-M-tile counter; the TMA producer issues A loads for a tile
//            only when its counter shows all remote rows present.  Tiles run local-rows-first, so the
//            pull overlaps the MMAs of the local tiles.
//   RS mode  C_partial = A B^T; the epilogue stores every output row straight into the receive slot
//            of the rank that owns it (bf16, 16-byte P2P stores), peer-owned tiles first, so the
//            reduce-scatter traffic overlaps the remaining MMAs.  The owner sums its slots after a
//            barrier (tp_sum_slots).
//
// Parity: Megatron sequence-parallel ColumnParallelLinear (all-gather -> GEMM) and
// RowParallelLinear (GEMM -> reduce-scatter) used by the reference's TP2 path
// (verl/models/mcore/tpr/attention.py:117-126, 195-221).
// ================================================================================================
namespace {

struct TpArgs {
  void* peer[8];          // AG: peers' staging [Ms, K]; RS: peers' receive buffers [n, Ms, N]
  int n, rank, Ms;
  int* counters;          // AG: rows copied per M-tile
  __nv_bfloat16* gather;  // AG: local A_full [M, K]
  long lda;               // AG: row stride (elements) of staging and A_full
  unsigned long long timeout_ns;
};

__device__ __forceinline__ uint64_t tp_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// remote rows of A that fall in M-tile mt (rows not owned by `rank`)
__device__ __forceinline__ int tp_expected(int mt, int M, int Ms, int rank) {
  const int lo = mt * BM, hi = min(M, lo + BM);
  const int own_lo = max(lo, rank * Ms), own_hi = min(hi, (rank + 1) * Ms);
  return (hi - lo) - max(0, own_hi - own_lo);
}

template <int MODE, bool B_MN>  // MODE 1: all-gather A then GEMM; MODE 2: GEMM then reduce-scatter rows
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tp_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, void* C,
                   int M, int N, int K, long ldc, int* err, const __grid_constant__ TpArgs tp) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem + SmemLayout::A_OFF;
  unsigned char* sB = smem + SmemLayout::B_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int nk = (K + BK - 1) / BK;
  // first M-tile in the schedule: the local shard (AG) or the next rank's shard (RS)
  const int first_row = MODE == 1 ? tp.rank * tp.Ms : ((tp.rank + 1) % tp.n) * tp.Ms;
  const int shift = min(first_row / BM, m_tiles - 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tfull[a], 1);
      sm100::mbar_init(&tempty[a], 128);
    }
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tmap_a);
    sm100::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, TMEM_COLS);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto tile_coords = [&](int t, int& m0, int& n0, int& mt) {
    const int group = 8;
    const int per_group = group * n_tiles;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gm = min(group, m_tiles - first_m);
    const int r = t % per_group;
    mt = (first_m + r % gm + shift) % m_tiles;
    m0 = mt * BM;
    n0 = (r / gm) * BN;
  };

  constexpr uint32_t IDESC = sm100::umma_idesc_bf16(BM, BN, false, B_MN);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int ready_mt = -1;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int m0, n0, mt;
        tile_coords(t, m0, n0, mt);
        if (MODE == 1 && mt != ready_mt) {
          const int want = tp_expected(mt, M, tp.Ms, tp.rank);
          const uint64_t t0 = tp_now();
          while (ld_acquire_gpu(tp.counters + mt) < want) {
            if (tp_now() - t0 > tp.timeout_ns) {
              atomicCAS(err, 0, 20);
              ok = false;
              break;
            }
            __nanosleep(128);
          }
          if (!ok) break;
          asm volatile("fence.proxy.async.global;" ::: "memory");
          ready_mt = mt;
        }
        for (int kb = 0; kb < nk; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1, err, 1)) {
            ok = false;
            break;
          }
          sm100::mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          unsigned char* a_dst = sA + stage * A_BYTES;
          unsigned char* b_dst = sB + stage * B_BYTES;
          sm100::tma_load_2d(a_dst, &tmap_a, &full[stage], kb * BK, m0);
          if (B_MN) {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              sm100::tma_load_2d(b_dst + i * 8192, &tmap_b, &full[stage], n0 + 64 * i, kb * BK);
          } else {
            sm100::tma_load_2d(b_dst, &tmap_b, &full[stage], kb * BK, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!sm100::mbar_wait(&tempty[acc], acc_phase ^ 1, err, 2)) break;
        sm100::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!sm100::mbar_wait(&full[stage], phase, err, 3)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_base = sm100::smem_addr(sA + stage * A_BYTES);
          const uint32_t b_base = sm100::smem_addr(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = sm100::umma_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sm100::umma_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                     : sm100::umma_desc_sw128(b_base + kk * 32, 16, 1024);
            sm100::umma_bf16(d_tmem, ad, bd, IDESC, (kb | kk) != 0);
          }
          sm100::umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        sm100::umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    if (MODE == 1) {
      // ---- pull the peers' rows of A into the local gather buffer, local-first tile order
      const int gw = blockIdx.x * 4 + (warp - 2), nw = gridDim.x * 4;
      const int vecs = K / 8;
      for (int idx = gw; idx < M; idx += nw) {
        const int row = (idx + tp.rank * tp.Ms) % M;
        const int owner = min(row / tp.Ms, tp.n - 1);
        if (owner == tp.rank) continue;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(tp.peer[owner]) +
                                                          (size_t)(row - owner * tp.Ms) * tp.lda);
        uint4* dst = reinterpret_cast<uint4*>(tp.gather + (size_t)row * tp.lda);
        // 8 independent 16-byte NVLink loads in flight per lane, then the local stores
        for (int v0 = 0; v0 < vecs; v0 += 32 * 8) {
          uint4 buf[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int v = v0 + u * 32 + lane;
            if (v < vecs) buf[u] = __ldg(src + v);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int v = v0 + u * 32 + lane;
            if (v < vecs) dst[v] = buf[u];
          }
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(tp.counters + row / BM, 1);
      }
    }
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int m0, n0, mt;
      tile_coords(t, m0, n0, mt);
      const bool got = sm100::mbar_wait(&tfull[acc], acc_phase, err, 4);
      if (!__all_sync(0xffffffffu, got)) break;
      sm100::tc_fence_after();
      const int row = m0 + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (MODE == 2) {
        // 32 rows x 64 columns per pass through a per-warp shared tile; lane groups of 8 then write
        // 128 contiguous bytes of one row each (4 rows per store instruction) to the row's owner.
        uint32_t* stile = reinterpret_cast<uint32_t*>(smem + SmemLayout::EPI_OFF) + (warp - 2) * (32 * 33);
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t r[32], r2[32];
          sm100::tmem_ld32(t_row + c * 64, r);
          sm100::tmem_ld32(t_row + c * 64 + 32, r2);
          sm100::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
            __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(r2[2 * j]), __uint_as_float(r2[2 * j + 1]));
            stile[lane * 33 + j] = *reinterpret_cast<uint32_t*>(&h);
            stile[lane * 33 + 16 + j] = *reinterpret_cast<uint32_t*>(&h2);
          }
          __syncwarp();
          const int col0 = n0 + c * 64;
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);    // tile row handled by this lane group
            const int part = lane & 7;              // 16-byte part of the 128-byte row segment
            const int grow = m0 + quarter * 32 + rr;
            const int col = col0 + part * 8;
            if (grow < M && col < N) {
              const int owner = min(grow / tp.Ms, tp.n - 1);
              __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(tp.peer[owner]) +
                                   ((size_t)tp.rank * tp.Ms + (grow - owner * tp.Ms)) * (size_t)N + col;
              const uint32_t* srow = stile + rr * 33 + part * 4;
              if (col + 8 <= N) {
                *reinterpret_cast<uint4*>(dst) = make_uint4(srow[0], srow[1], srow[2], srow[3]);
              } else {
                const __nv_bfloat16* hs = reinterpret_cast<const __nv_bfloat16*>(srow);
                for (int e = 0; e < 8 && col + e < N; ++e) dst[e] = hs[e];
              }
            }
          }
          __syncwarp();
        }
      } else {
        __nv_bfloat16* dst_row = row < M ? reinterpret_cast<__nv_bfloat16*>(C) + (size_t)row * ldc : nullptr;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(t_row + c * 32, r);
          sm100::tmem_ld_wait();
          const int col0 = n0 + c * 32;
          if (dst_row && col0 < N) {
            __nv_bfloat16* dst = dst_row + col0;
            if (col0 + 32 <= N) {
              uint32_t p[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                p[j] = *reinterpret_cast<uint32_t*>(&h);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(dst)[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
            } else {
              for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] = __float2bfloat16(__uint_as_float(r[j]));
            }
          }
        }
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int MODE, bool B_MN>
void tp_launch(const MapPair* maps, void* c, int M, int N, int K, long ldc, const TpArgs& tp) {
  auto kern = tp_gemm_kernel<MODE, B_MN>;
  const int smem = (MODE == 2 ? SmemLayout::TOTAL_EPI : SmemLayout::TOTAL) + 1024;
  static unsigned long long attr_done = 0;
  bb::set_smem_attr_once(kern, smem, attr_done);
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  // AG: every CTA must be resident (CTAs wait on rows copied by other CTAs): at most one per SM
  const int grid = std::max(1, std::min(tiles, num_sms()));
  int* err = error_word().data_ptr<int>();
  void* args[] = {const_cast<CUtensorMap*>(&maps->a), const_cast<CUtensorMap*>(&maps->b), &c, &M, &N, &K, &ldc,
                  &err, const_cast<TpArgs*>(&tp)};
  BB_CHECK_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(NUM_THREADS), args, smem,
                                 at::cuda::getCurrentCUDAStream()));
  BB_POST_LAUNCH();
}

__global__ void tp_sum_slots_kernel(const uint4* __restrict__ recv, uint4* __restrict__ out, int n, size_t vecs) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < vecs; i += stride) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < n; ++s) {
      bb::bf16x8 v = reinterpret_cast<const bb::bf16x8*>(recv)[(size_t)s * vecs + i];
      float f[8];
      bb::unpack8(v, f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
    reinterpret_cast<bb::bf16x8*>(out)[i] = bb::pack8(acc);
  }
}

TpArgs make_tp_args(const std::vector<int64_t>& peers, int64_t rank, int64_t ms, double timeout_s) {
  TORCH_CHECK(!peers.empty() && peers.size() <= 8, "tp gemm: 1..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < (int64_t)peers.size() && ms > 0, "tp gemm: bad rank / rows per rank");
  TpArgs tp{};
  for (size_t i = 0; i < peers.size(); ++i) {
    TORCH_CHECK(peers[i] % 16 == 0, "tp gemm: peer buffers must be 16-byte aligned");
    tp.peer[i] = reinterpret_cast<void*>(peers[i]);
  }
  tp.n = (int)peers.size();
  tp.rank = (int)rank;
  tp.Ms = (int)ms;
  tp.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  return tp;
}

void tp_context(int dev) {
  at::cuda::CUDAGuard guard(dev);
  CUcontext cur = nullptr;
  if (cuCtxGetCurrent(&cur) != CUDA_SUCCESS || cur == nullptr) BB_CHECK_CUDA(cudaFree(nullptr));
}

}  // namespace

// AG + GEMM: `gather` [M, K] bf16 holds this rank's rows already; the kernel pulls the others from the
// peers' staging buffers (`peers[j]` = rank j's [Ms, K] staging) and returns C = gather @ op(B)^T.
torch::Tensor tp_ag_gemm(torch::Tensor gather, torch::Tensor b, bool b_mn, std::vector<int64_t> peers, int64_t rank,
                         int64_t ms, torch::Tensor counters, double timeout_s) {
  TORCH_CHECK(gather.is_cuda() && gather.scalar_type() == at::kBFloat16 && gather.is_contiguous(), "tp_ag_gemm: A");
  TORCH_CHECK(b.scalar_type() == at::kBFloat16 && b.stride(1) == 1, "tp_ag_gemm: B");
  const long M = gather.size(0), K = gather.size(1);
  const long N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K && K % 8 == 0 && b.stride(0) % 8 == 0, "tp_ag_gemm: shapes");
  TORCH_CHECK(M <= (long)ms * (long)peers.size(), "tp_ag_gemm: M exceeds ranks x rows per rank");
  const int m_tiles = (int)((M + BM - 1) / BM);
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= m_tiles,
              "tp_ag_gemm: counters");
  auto c = torch::empty({M, N}, gather.options());
  tp_context(gather.get_device());
  counters.zero_();
  TpArgs tp = make_tp_args(peers, rank, ms, timeout_s);
  tp.counters = counters.data_ptr<int>();
  tp.gather = reinterpret_cast<__nv_bfloat16*>(gather.data_ptr());
  tp.lda = K;
  MapPair* maps = map_storage();
  make_map(&maps->a, gather.data_ptr(), M, K, K, BM);
  if (b_mn) make_map(&maps->b, b.data_ptr(), K, N, b.stride(0), 64);
  else make_map(&maps->b, b.data_ptr(), N, K, b.stride(0), BN);
  if (b_mn) tp_launch<1, true>(maps, c.data_ptr(), (int)M, (int)N, (int)K, N, tp);
  else tp_launch<1, false>(maps, c.data_ptr(), (int)M, (int)N, (int)K, N, tp);
  return c;
}

// GEMM + RS: C_partial = A @ op(B)^T with row r stored into the receive buffer of rank r / Ms,
// slot `rank` (`peers[j]` = rank j's [n, Ms, N] bf16 receive buffer).
void tp_gemm_rs(torch::Tensor a, torch::Tensor b, bool b_mn, std::vector<int64_t> peers, int64_t rank, int64_t ms,
                double timeout_s) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && a.stride(1) == 1 && a.stride(0) % 8 == 0,
              "tp_gemm_rs: A");
  TORCH_CHECK(b.scalar_type() == at::kBFloat16 && b.stride(1) == 1 && b.stride(0) % 8 == 0, "tp_gemm_rs: B");
  const long M = a.size(0), K = a.size(1);
  const long N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K && N % 8 == 0, "tp_gemm_rs: shapes (N must be a multiple of 8)");
  TORCH_CHECK(M <= (long)ms * (long)peers.size(), "tp_gemm_rs: M exceeds ranks x rows per rank");
  if (M == 0 || N == 0) return;
  tp_context(a.get_device());
  TpArgs tp = make_tp_args(peers, rank, ms, timeout_s);
  MapPair* maps = map_storage();
  make_map(&maps->a, a.data_ptr(), M, K, a.stride(0), BM);
  if (b_mn) make_map(&maps->b, b.data_ptr(), K, N, b.stride(0), 64);
  else make_map(&maps->b, b.data_ptr(), N, K, b.stride(0), BN);
  if (b_mn) tp_launch<2, true>(maps, nullptr, (int)M, (int)N, (int)K, N, tp);
  else tp_launch<2, false>(maps, nullptr, (int)M, (int)N, (int)K, N, tp);
}

// out[Ms, N] = sum over the n slots of recv[n, Ms, N] (FP32 accumulation, bf16 out)
torch::Tensor tp_sum_slots(torch::Tensor recv, int64_t n, int64_t ms, int64_t N) {
  TORCH_CHECK(recv.is_cuda() && recv.scalar_type() == at::kBFloat16 && recv.numel() >= n * ms * N && N % 8 == 0,
              "tp_sum_slots: recv");
  auto out = torch::empty({ms, N}, recv.options());
  const size_t vecs = (size_t)ms * N / 8;
  const int blocks = (int)std::min<size_t>((vecs + 255) / 256, (size_t)num_sms() * 8);
  tp_sum_slots_kernel<<<std::max(blocks, 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(recv.data_ptr()), reinterpret_cast<uint4*>(out.data_ptr()), (int)n, vecs);
  BB_POST_LAUNCH();
  return out;
}

// ================================================================================================
// Grouped (mixture-of-experts) tcgen05 GEMMs with device-side expert offsets (no host sync):
//
//   MODE 0  out[off_e + i, :] = x[off_e + i, :] @ W[e]^T        W as [E*N, K]   (forward)
//   MODE 1  out[off_e + i, :] = x[off_e + i, :] @ W[e]          W as [E*K', N]  (data gradient;
//                                                                K' % 64 == 0, MN-major B)
//   MODE 2  acc[e] += dy[rows_e, :]^T @ x[rows_e, :]           FP32 [E, M, N]  (weight gradient;
//                                                                K = the expert's token rows)
// Rows of one expert are contiguous (tokens sorted by expert); offsets int32 [E+1] live on the
// device.  Each CTA scans the offsets into shared memory and walks the same persistent tile list
// as the plain GEMM.  In MODE 2 the last K block of an expert also covers the next expert's rows:
// the MMA warp zeroes those rows of the A stage in shared memory (generic stores, then a proxy
// fence) before issuing the MMAs, so only the expert's own tokens contribute.
// ================================================================================================
namespace {

constexpr int kMaxExperts = 1024;

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, void* C,
                        const int* __restrict__ offsets, int E, int N, int K, long ldc, int* err) {
  // MODE 0/1: N = output columns, K = reduction dim (per-expert weight rows for MODE 1).
  // MODE 2  : N = output columns (x width), K unused (rows per expert from offsets); M = ldc rows per expert.
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem + SmemLayout::A_OFF;
  unsigned char* sB = smem + SmemLayout::B_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  int* pre = reinterpret_cast<int*>(smem + SmemLayout::BAR_OFF + 256);   // [E+1] prefix of M tiles

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (N + BN - 1) / BN;
  const int Mrows = (int)ldc;  // MODE 2: rows of one expert's output (= out features)
  const int m2_tiles = (Mrows + BM - 1) / BM;

  if (threadIdx.x == 0) {
    int acc = 0;
    pre[0] = 0;
    for (int e = 0; e < E; ++e) {
      const int rows = offsets[e + 1] - offsets[e];
      acc += MODE == 2 ? (rows > 0 ? m2_tiles : 0) : (rows + BM - 1) / BM;
      pre[e + 1] = acc;
    }
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tfull[a], 1);
      sm100::mbar_init(&tempty[a], 128);
    }
    sm100::fence_mbar_init();
    sm100::prefetch_tmap(&tmap_a);
    sm100::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, TMEM_COLS);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = pre[E] * n_tiles;

  // tile t -> expert e, M tile mt (within the expert), N tile nt
  auto tile_of = [&](int t, int& e, int& m0, int& n0) {
    const int mt_global = t / n_tiles;
    int lo = 0, hi = E - 1;
    while (lo < hi) {  // last e with pre[e] <= mt_global
      const int mid = (lo + hi + 1) >> 1;
      if (pre[mid] <= mt_global) lo = mid;
      else hi = mid - 1;
    }
    e = lo;
    m0 = (mt_global - pre[e]) * BM;
    n0 = (t % n_tiles) * BN;
  };
  auto kblocks = [&](int e) {
    return MODE == 2 ? (offsets[e + 1] - offsets[e] + BK - 1) / BK : (K + BK - 1) / BK;
  };

  constexpr bool A_MN = MODE == 2;
  constexpr bool B_MN = MODE != 0;
  constexpr uint32_t IDESC = sm100::umma_idesc_bf16(BM, BN, A_MN, B_MN);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int e, m0, n0;
        tile_of(t, e, m0, n0);
        const int nk = kblocks(e);
        const int row0 = offsets[e];
        for (int kb = 0; kb < nk; ++kb) {
          if (!sm100::mbar_wait(&empty[stage], phase ^ 1, err, 1)) {
            ok = false;
            break;
          }
          sm100::mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          unsigned char* a_dst = sA + stage * A_BYTES;
          unsigned char* b_dst = sB + stage * B_BYTES;
          if (MODE == 2) {
            // A = dy^T: MN-major tile of dy rows [row0 + kb*64, +64), columns [m0, m0+128)
#pragma unroll
            for (int i = 0; i < BM / 64; ++i)
              sm100::tma_load_2d(a_dst + i * 8192, &tmap_a, &full[stage], m0 + 64 * i, row0 + kb * BK);
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              sm100::tma_load_2d(b_dst + i * 8192, &tmap_b, &full[stage], n0 + 64 * i, row0 + kb * BK);
          } else {
            sm100::tma_load_2d(a_dst, &tmap_a, &full[stage], kb * BK, row0 + m0);
            if (MODE == 1) {
#pragma unroll
              for (int i = 0; i < BN / 64; ++i)
                sm100::tma_load_2d(b_dst + i * 8192, &tmap_b, &full[stage], n0 + 64 * i, e * K + kb * BK);
            } else {
              sm100::tma_load_2d(b_dst, &tmap_b, &full[stage], kb * BK, e * N + n0);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      int e, m0, n0;
      tile_of(t, e, m0, n0);
      const int nk = kblocks(e);
      const int rows_e = offsets[e + 1] - offsets[e];
      // every lane waits; decisions are warp-uniform so the whole warp leaves together
      if (!__all_sync(0xffffffffu, sm100::mbar_wait(&tempty[acc], acc_phase ^ 1, err, 2))) break;
      sm100::tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < nk; ++kb) {
        if (!__all_sync(0xffffffffu, sm100::mbar_wait(&full[stage], phase, err, 3))) {
          ok = false;
          break;
        }
        if (MODE == 2) {
          const int valid = rows_e - kb * BK;  // token rows of this expert in the block
          if (valid < BK) {
            // zero K rows [valid, 64) of the A stage: each 8 KB chunk holds 64 rows of 128 bytes
            unsigned char* a_st = sA + stage * A_BYTES;
            const int nrows = BK - valid;
            for (int i = lane; i < (BM / 64) * nrows * 8; i += 32) {
              const int chunk = i / (nrows * 8), rem = i % (nrows * 8);
              const int r = valid + rem / 8, part = rem % 8;
              *reinterpret_cast<uint4*>(a_st + chunk * 8192 + r * 128 + part * 16) = make_uint4(0, 0, 0, 0);
            }
            sm100::fence_proxy_async_smem();
            __syncwarp();
          }
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t a_base = sm100::smem_addr(sA + stage * A_BYTES);
          const uint32_t b_base = sm100::smem_addr(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sm100::umma_desc_sw128(a_base + kk * 2048, 8192, 1024)
                                     : sm100::umma_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sm100::umma_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                     : sm100::umma_desc_sw128(b_base + kk * 32, 16, 1024);
            sm100::umma_bf16(d_tmem, ad, bd, IDESC, (kb | kk) != 0);
          }
          sm100::umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) sm100::umma_commit(&tfull[acc]);
      __syncwarp();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  } else {
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int e, m0, n0;
      tile_of(t, e, m0, n0);
      const bool got = sm100::mbar_wait(&tfull[acc], acc_phase, err, 4);
      if (!__all_sync(0xffffffffu, got)) break;
      sm100::tc_fence_after();
      const int r = m0 + quarter * 32 + lane;  // row within the expert's output block
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const int rows_lim = MODE == 2 ? Mrows : offsets[e + 1] - offsets[e];
      const bool row_ok = r < rows_lim;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        sm100::tmem_ld32(t_row + c * 32, v);
        sm100::tmem_ld_wait();
        const int col0 = n0 + c * 32;
        if (!row_ok || col0 >= N) continue;
        if (MODE == 2) {
          float* dst = reinterpret_cast<float*>(C) + ((size_t)e * Mrows + r) * (size_t)N + col0;
          if (col0 + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4 a = reinterpret_cast<float4*>(dst)[j];
              a.x += __uint_as_float(v[4 * j]);
              a.y += __uint_as_float(v[4 * j + 1]);
              a.z += __uint_as_float(v[4 * j + 2]);
              a.w += __uint_as_float(v[4 * j + 3]);
              reinterpret_cast<float4*>(dst)[j] = a;
            }
          } else {
            for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] += __uint_as_float(v[j]);
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (size_t)(offsets[e] + r) * (size_t)N + col0;
          if (col0 + 32 <= N) {
            uint32_t p[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
              p[j] = *reinterpret_cast<uint32_t*>(&h);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
              reinterpret_cast<uint4*>(dst)[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
          } else {
            for (int j = 0; j < 32 && col0 + j < N; ++j) dst[j] = __float2bfloat16(__uint_as_float(v[j]));
          }
        }
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int MODE>
void grouped_launch(const MapPair* maps, void* c, const int* offsets, int E, int N, int K, long ldc, int grid) {
  auto kern = grouped_gemm_kernel<MODE>;
  const int smem = SmemLayout::TOTAL + 4 * (kMaxExperts + 1) + 1024;
  static unsigned long long attr_done = 0;
  bb::set_smem_attr_once(kern, smem, attr_done);
  int* err = error_word().data_ptr<int>();
  void* args[] = {const_cast<CUtensorMap*>(&maps->a), const_cast<CUtensorMap*>(&maps->b), &c,
                  const_cast<int**>(&offsets), &E, &N, &K, &ldc, &err};
  BB_CHECK_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(NUM_THREADS), args, smem,
                                 at::cuda::getCurrentCUDAStream()));
  BB_POST_LAUNCH();
}

}  // namespace

// x [T, K] rows sorted by expert, offsets int32 [E+1] (device), w [E, N, K] (trans_w=false: out = x W_e^T)
// or w [E, K, N] (trans_w=true: out = x W_e).  Returns bf16 [T, N].
torch::Tensor grouped_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor offsets, bool trans_w) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "grouped: x");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 3, "grouped: w [E, rows, cols]");
  TORCH_CHECK(offsets.is_cuda() && offsets.scalar_type() == at::kInt && offsets.numel() == w.size(0) + 1,
              "grouped: offsets int32 [E+1] on the device");
  const int E = (int)w.size(0);
  TORCH_CHECK(E <= kMaxExperts, "grouped: at most 1024 experts");
  const long T = x.size(0), K = x.size(1);
  const long N = trans_w ? w.size(2) : w.size(1);
  TORCH_CHECK((trans_w ? w.size(1) : w.size(2)) == K, "grouped: inner dimensions differ");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "grouped: K and N must be multiples of 8");
  if (trans_w) TORCH_CHECK(K % BK == 0, "grouped: the reduction dim of a transposed expert weight must be % 64");
  auto out = torch::empty({T, N}, x.options());
  if (T == 0 || N == 0) return out;
  tp_context(x.get_device());
  MapPair* maps = map_storage();
  make_map(&maps->a, x.data_ptr(), T, K, K, BM);
  if (trans_w) make_map(&maps->b, w.data_ptr(), (long)E * K, N, N, 64);
  else make_map(&maps->b, w.data_ptr(), (long)E * N, K, K, BN);
  const long n_tiles = (N + BN - 1) / BN;
  const int grid = (int)std::max<long>(1, std::min<long>((T / BM + E) * n_tiles, num_sms()));
  if (trans_w) grouped_launch<1>(maps, out.data_ptr(), offsets.data_ptr<int>(), E, (int)N, (int)K, N, grid);
  else grouped_launch<0>(maps, out.data_ptr(), offsets.data_ptr<int>(), E, (int)N, (int)K, N, grid);
  return out;
}

// acc [E, M, N] FP32 += per expert dy[rows_e]^T @ x[rows_e] with dy [T, M], x [T, N] (rows sorted by expert).
void grouped_gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor offsets, torch::Tensor acc) {
  TORCH_CHECK(dy.is_cuda() && dy.scalar_type() == at::kBFloat16 && dy.is_contiguous(), "grouped wgrad: dy");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.size(0) == dy.size(0), "grouped wgrad: x");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.dim() == 3, "grouped wgrad: acc");
  const int E = (int)acc.size(0);
  TORCH_CHECK(E <= kMaxExperts && offsets.numel() == E + 1 && offsets.scalar_type() == at::kInt, "grouped wgrad: E");
  const long T = dy.size(0), M = dy.size(1), N = x.size(1);
  TORCH_CHECK(acc.size(1) == M && acc.size(2) == N && M % 8 == 0 && N % 8 == 0, "grouped wgrad: shapes");
  if (T == 0) return;
  tp_context(dy.get_device());
  MapPair* maps = map_storage();
  make_map(&maps->a, dy.data_ptr(), T, M, M, 64);
  make_map(&maps->b, x.data_ptr(), T, N, N, 64);
  const long tiles = (long)E * ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = (int)std::max<long>(1, std::min<long>(tiles, num_sms()));
  grouped_launch<2>(maps, acc.data_ptr(), offsets.data_ptr<int>(), E, (int)N, 0, M, grid);
}
