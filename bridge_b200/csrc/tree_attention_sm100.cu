// tcgen05 / TMEM flash-attention forward for the tree (prefix-reuse) layout, head_dim 128.
//
// One CTA = 128 query rows of one sequence x one q head.  Key tiles of 128: first the sequence's
// prefix span in the bank (full visibility), then its own keys up to the tile's last query (causal).
//
//   warp 0      TMA producer: Q once (2 boxes), then K/V tiles into a 2-stage ring
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer:
//                 S_j = Q K_j^T  -> TMEM S[j%2]     (issued before PV_{j-1}, so it overlaps softmax_{j-1})
//                 O  += P_j V_j  -> TMEM O          (A = P from swizzled smem, B = V MN-major)
//   warps 2-5   softmax (one thread per query row): tcgen05.ld S, mask, online softmax in the exp2
//               domain with a lazily updated reference max (O is rescaled in TMEM only when the row max
//               grows by more than 2^8), P -> smem (128-byte swizzle), epilogue O / l -> bf16, LSE.
//               P is double-buffered, so the exponentials of tile j run while P_{j-1} V_{j-1} is on the
//               tensor cores (only a rescale of O waits for that product); tiles whose every key is
//               visible to every row skip the mask, and the softmax scale is folded into the exponent.
//
// TMEM: S0 | S1 | O = 384 of 512 columns.  Shared memory: Q 32 KB + 2 x (K 32 KB + V 32 KB) + 2 x P 32 KB.
// All waits are bounded (sm100_common.cuh).
#include <torch/extension.h>
#include <string>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "sm100_common.cuh"

namespace {

constexpr int D = 128;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int TILE_BYTES = BQ * D * 2;  // 32 KB (two 64-column swizzle blocks of 16 KB)
constexpr int NUM_THREADS = 192;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

struct Smem {
  static constexpr int Q = 0;
  static constexpr int K0 = Q + TILE_BYTES;
  static constexpr int V0 = K0 + 2 * TILE_BYTES;
  static constexpr int P = V0 + 2 * TILE_BYTES;   // [2] P tiles
  static constexpr int BAR = P + 2 * TILE_BYTES;
  static constexpr int TOTAL = BAR + 256;
};
static_assert(Smem::TOTAL + 1024 <= 232448, "forward shared memory above the 227 KB per-block limit");

// Optional phase timing of the forward (a profiling aid, off unless attn_phase_profile(true)): the first
// softmax thread of each CTA adds the SM cycles from kernel entry to the first S tile, of the tile loop
// and of the epilogue, plus its tile count: g_attn_prof = {startup, loop, epilogue, tiles, ctas}.
__device__ int g_attn_prof_on;
__device__ unsigned long long g_attn_prof[8];

struct alignas(64) AttnMaps {
  CUtensorMap q, k, v, pk, pv;
};

__device__ __forceinline__ void load_tile128(unsigned char* dst, const CUtensorMap* map, uint64_t* bar, int col0,
                                             int row0) {
  sm100::tma_load_2d(dst, map, bar, col0, row0);
  sm100::tma_load_2d(dst + 16384, map, bar, col0 + 64, row0);
}

// K-major SW128 descriptor for a [128 rows x 128] bf16 tile stored as two 64-column blocks, k-step kk (16 elems).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return sm100::umma_desc_sw128(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
// MN-major SW128 descriptor for V [128 keys (K) x 128 d (N)] stored as two 64-d blocks of 128 rows.
__device__ __forceinline__ uint64_t vmajor_desc(uint32_t base, int kk) {
  return sm100::umma_desc_sw128(base + kk * 2048, 16384, 1024);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    tree_attn_fwd_sm100_kernel(const __grid_constant__ AttnMaps maps, const int* __restrict__ cu,
                               const int* __restrict__ poff, const int* __restrict__ plen,
                               __nv_bfloat16* __restrict__ out, float* __restrict__ lse, int T, int Hq, int Hk,
                               float scale_log2, int* err) {
  const int seq = blockIdx.y, h = blockIdx.z, hk = h / (Hq / Hk);
  const int q0 = cu[seq], n = cu[seq + 1] - q0;
  const int m0 = blockIdx.x * BQ;
  if (m0 >= n) return;  // before any TMEM/barrier work
  const bool prof = threadIdx.x == 64 && g_attn_prof_on != 0;
  long long t_entry = prof ? clock64() : 0, t_first = 0;
  const int po = poff[seq], pl = plen[seq];
  const int n_pre = (pl + BKV - 1) / BKV;
  const int n_self_keys = min(n, m0 + BQ);
  const int n_self = (n_self_keys + BKV - 1) / BKV;
  const int ntiles = n_pre + n_self;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::BAR);
  uint64_t* bar_q = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;    // [2] P_j written (softmax -> MMA)
  uint64_t* p_free = bars + 11;   // [2] P_j V_j done: P buffer reusable, O holds tiles <= j
  uint64_t* o_done = bars + 13;   // the last P V done (epilogue)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sm100::mbar_init(bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&kv_full[i], 1);
      sm100::mbar_init(&kv_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&s_free[i], 128);
      sm100::mbar_init(&p_full[i], 128);
      sm100::mbar_init(&p_free[i], 1);
    }
    sm100::mbar_init(o_done, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_S0 = tmem, TM_O = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      sm100::mbar_expect_tx(bar_q, TILE_BYTES);
      load_tile128(smem + Smem::Q, &maps.q, bar_q, h * D, q0 + m0);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        if (!sm100::mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, err, 11)) break;
        sm100::mbar_expect_tx(&kv_full[st], 2 * TILE_BYTES);
        const bool pre = j < n_pre;
        const int row = pre ? po + j * BKV : q0 + (j - n_pre) * BKV;
        load_tile128(smem + Smem::K0 + st * TILE_BYTES, pre ? &maps.pk : &maps.k, &kv_full[st], hk * D, row);
        load_tile128(smem + Smem::V0 + st * TILE_BYTES, pre ? &maps.pv : &maps.v, &kv_full[st], hk * D, row);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = sm100::umma_idesc_bf16(BQ, BKV, false, false);
      constexpr uint32_t IDESC_O = sm100::umma_idesc_bf16(BQ, D, false, true);
      const uint32_t q_base = sm100::smem_addr(smem + Smem::Q);
      const uint32_t p_base = sm100::smem_addr(smem + Smem::P);
      bool ok = sm100::mbar_wait(bar_q, 0, err, 12);
      auto issue_pv = [&](int j) -> bool {
        if (!sm100::mbar_wait(&p_full[j & 1], (j >> 1) & 1, err, 13)) return false;
        sm100::tc_fence_after();
        const uint32_t v_base = sm100::smem_addr(smem + Smem::V0 + (j & 1) * TILE_BYTES);
        const uint32_t pj = p_base + (j & 1) * TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          sm100::umma_bf16(TM_O, kmajor_desc(pj, kk), vmajor_desc(v_base, kk), IDESC_O, (j > 0 || kk > 0));
        sm100::umma_commit(&p_free[j & 1]);
        sm100::umma_commit(&kv_empty[j & 1]);
        if (j == ntiles - 1) sm100::umma_commit(o_done);
        return true;
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        const int st = j & 1;
        if (!sm100::mbar_wait(&kv_full[st], (j >> 1) & 1, err, 14)) {
          ok = false;
          break;
        }
        if (!sm100::mbar_wait(&s_free[st], ((j >> 1) & 1) ^ 1, err, 15)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t k_base = sm100::smem_addr(smem + Smem::K0 + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          sm100::umma_bf16(TM_S0 + st * BKV, kmajor_desc(q_base, kk), kmajor_desc(k_base, kk), IDESC_S, kk > 0);
        sm100::umma_commit(&s_full[st]);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(ntiles - 1);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;       // TMEM lane == query row within the tile
    const int qi = m0 + row;                   // local query index
    const bool row_ok = qi < n;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    unsigned char* sP = smem + Smem::P;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int st = j & 1;
      const bool got = sm100::mbar_wait(&s_full[st], (j >> 1) & 1, err, 16);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      if (prof && j == 0) t_first = clock64();
      sm100::tc_fence_after();
      // the four 32-column loads in flight together, one wait
      uint32_t r0[32], r1[32], r2[32], r3[32];
      const uint32_t ts = TM_S0 + st * BKV + lane_off;
      sm100::tmem_ld32(ts, r0);
      sm100::tmem_ld32(ts + 32, r1);
      sm100::tmem_ld32(ts + 64, r2);
      sm100::tmem_ld32(ts + 96, r3);
      sm100::tmem_ld_wait();
      sm100::tmem_regs_ready(r0);
      sm100::tmem_regs_ready(r1);
      sm100::tmem_regs_ready(r2);
      sm100::tmem_regs_ready(r3);
      sm100::tc_fence_before();
      sm100::mbar_arrive(&s_free[st]);  // S buffer may be overwritten by S_{j+2}
      float s[BKV];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        s[e] = __uint_as_float(r0[e]);
        s[32 + e] = __uint_as_float(r1[e]);
        s[64 + e] = __uint_as_float(r2[e]);
        s[96 + e] = __uint_as_float(r3[e]);
      }
      // keys [kb, klim) are visible to this row; a tile wholly inside every row's range skips the mask
      const bool pre = j < n_pre;
      const int kb = pre ? j * BKV : (j - n_pre) * BKV;
      const int klim = pre ? pl : min(n, qi + 1);
      float mx = -INFINITY;
      if (__all_sync(0xffffffffu, row_ok && kb + BKV <= klim)) {
#pragma unroll
        for (int e = 0; e < BKV; ++e) mx = fmaxf(mx, s[e]);
      } else {
#pragma unroll
        for (int e = 0; e < BKV; ++e) {
          const float x = (row_ok && (kb + e) < klim) ? s[e] : -INFINITY;
          s[e] = x;
          mx = fmaxf(mx, x);
        }
      }
      mx *= scale_log2;   // scale > 0: the max of the scaled scores
      // lazily updated reference max
      float alpha = 1.f;
      if (mx > m_ref + RESCALE_THRESHOLD || (m_ref == -INFINITY && mx > -INFINITY)) {
        const float m_new = mx;
        alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - m_new);
        m_ref = m_new;
      }
      // P buffer j & 1 was read by P_{j-2} V_{j-2}
      if (j >= 2) {
        const bool g1 = sm100::mbar_wait(&p_free[st], ((j >> 1) - 1) & 1, err, 19);
        if (!__all_sync(0xffffffffu, g1)) {
          ok = false;
          break;
        }
      }
      float rs = 0.f;
      const float msafe = (m_ref == -INFINITY) ? 0.f : m_ref;
      unsigned char* sPj = sP + st * TILE_BYTES;
      // P -> smem, 128-byte swizzle: 16-byte chunk index XOR (row & 7) within each 64-key block
#pragma unroll
      for (int c = 0; c < BKV / 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = exp2f(fmaf(s[c * 8 + 2 * e], scale_log2, -msafe));
          const float p1 = exp2f(fmaf(s[c * 8 + 2 * e + 1], scale_log2, -msafe));
          rs += p0 + p1;
          __nv_bfloat162 hv = __floats2bfloat162_rn(p0, p1);
          pk[e] = *reinterpret_cast<uint32_t*>(&hv);
        }
        const int blk = c >> 3, chunk = c & 7;
        unsigned char* dst = sPj + blk * 16384 + row * 128 + ((chunk ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l = l * alpha + rs;
      // a new reference max: O (tiles < j) is rescaled once P_{j-1} V_{j-1} has landed, before P_j V_j
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        const int jp = j - 1;
        const bool g2 = sm100::mbar_wait(&p_free[jp & 1], (jp >> 1) & 1, err, 17);
        if (!__all_sync(0xffffffffu, g2)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld32(TM_O + lane_off + c * 32, r);
          sm100::tmem_ld_wait();
          sm100::tmem_regs_ready(r);
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          sm100::tmem_st32(TM_O + lane_off + c * 32, r);
        }
        sm100::tmem_st_wait();
      }
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      sm100::mbar_arrive(&p_full[st]);
    }
    // epilogue
    const long long t_loop = prof ? clock64() : 0;
    const bool g3 = ok && sm100::mbar_wait(o_done, 0, err, 18);
    if (__all_sync(0xffffffffu, g3)) {
      sm100::tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const size_t qstride = (size_t)Hq * D;
      __nv_bfloat16* orow = out + (size_t)(q0 + qi) * qstride + (size_t)h * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(TM_O + lane_off + c * 32, r);
        sm100::tmem_ld_wait();
        if (row_ok) {
          uint32_t pkd[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            __nv_bfloat162 hv = __floats2bfloat162_rn(__uint_as_float(r[2 * e]) * inv, __uint_as_float(r[2 * e + 1]) * inv);
            pkd[e] = *reinterpret_cast<uint32_t*>(&hv);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e)
            reinterpret_cast<uint4*>(orow + c * 32)[e] = make_uint4(pkd[4 * e], pkd[4 * e + 1], pkd[4 * e + 2], pkd[4 * e + 3]);
        }
      }
      if (row_ok) lse[(size_t)h * T + q0 + qi] = l > 0.f ? (m_ref + log2f(l)) * 0.6931471805599453f : -INFINITY;
    }
    if (prof) {
      const long long t_end = clock64();
      atomicAdd(&g_attn_prof[0], (unsigned long long)(t_first - t_entry));
      atomicAdd(&g_attn_prof[1], (unsigned long long)(t_loop - t_first));
      atomicAdd(&g_attn_prof[2], (unsigned long long)(t_end - t_loop));
      atomicAdd(&g_attn_prof[3], (unsigned long long)ntiles);
      atomicAdd(&g_attn_prof[4], 1ull);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// =================================================================================== backward
// Backward = two tcgen05 kernels (no per-tile dQ atomics):
//   dkdv : one CTA = 128 keys x 1 kv head; loops over every (q head of the GQA group, 128-row q tile)
//          that sees them.  S^T = K Q^T and dP^T = V dO^T land in TMEM; the softmax warps (one thread per
//          key) form P^T and dS^T = P^T (dP^T - delta) in swizzled smem; dV += P^T dO, dK += dS^T Q
//          accumulate in TMEM across the loop.  Own keys: written once (bf16).  Prefix keys: the work is
//          split per reading sequence and merged with one vectorised FP32 atomic pass per CTA.
//   dq   : one CTA = 128 queries x 1 q head (forward-like loop over key tiles): S, dP in TMEM, dS -> smem,
//          dQ += dS K accumulated in TMEM, written once.
struct alignas(64) BwdMaps {
  CUtensorMap q, k, v, pk, pv, dout, q64, dout64;   // q64 / dout64: 64-row boxes for the pipelined dK/dV
  CUtensorMap k64, v64, pk64, pv64;                 // 64-row key / value boxes for the pipelined dQ
};

__device__ __forceinline__ void named_sync_softmax() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Barrier over the 4 softmax warps that also ANDs a predicate: every warp takes the same branch afterwards,
// so a bounded-wait failure in one warp can never leave the others waiting at a named barrier.
__device__ __forceinline__ bool named_and_softmax(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// Write 32 consecutive bf16-converted columns [c*32, c*32+32) of row `row` into a K-major SW128 tile.
__device__ __forceinline__ void store_row32_sw128(unsigned char* tile, int row, int c, const float* v) {
  uint32_t pk[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    pk[e] = *reinterpret_cast<uint32_t*>(&hv);
  }
  const int blk = c >> 1;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int chunk = (c & 1) * 4 + e;
    unsigned char* dst = tile + blk * 16384 + row * 128 + ((chunk ^ (row & 7)) << 4);
    *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
  }
}

struct SmemDKDV {
  static constexpr int K = 0;
  static constexpr int V = K + TILE_BYTES;
  static constexpr int Q = V + TILE_BYTES;
  static constexpr int DO = Q + TILE_BYTES;
  static constexpr int PT = DO + TILE_BYTES;
  static constexpr int DST = PT + TILE_BYTES;
  static constexpr int LSE = DST + TILE_BYTES;  // 128 floats
  static constexpr int DEL = LSE + 512;         // 128 floats
  static constexpr int BAR = DEL + 512;
  static constexpr int TOTAL = BAR + 256;
};

__global__ void __launch_bounds__(NUM_THREADS, 1)
    tree_attn_dkdv_sm100_kernel(const __grid_constant__ BwdMaps maps, const int* __restrict__ cu,
                                const int* __restrict__ poff, const int* __restrict__ plen,
                                const float* __restrict__ lse, const float* __restrict__ delta,
                                __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv,
                                float* __restrict__ dpk_acc, float* __restrict__ dpv_acc, int B, int T, int Hq,
                                int Hk, float scale_log2, float scale, int* err) {
  const int mode = blockIdx.y / B, b = blockIdx.y % B, hk = blockIdx.z, rep = Hq / Hk;
  const int q0 = cu[b], n = cu[b + 1] - q0;
  const int key_len = mode == 0 ? n : plen[b];
  const int key_row0 = mode == 0 ? q0 : poff[b];
  const int kb = blockIdx.x * BKV;
  if (kb >= key_len || n <= 0) return;
  const int it0 = mode == 0 ? kb / BQ : 0;
  const int nq = (n + BQ - 1) / BQ - it0;
  const int niter = rep * nq;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* lse_s = reinterpret_cast<float*>(smem + SmemDKDV::LSE);
  float* del_s = reinterpret_cast<float*>(smem + SmemDKDV::DEL);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemDKDV::BAR);
  uint64_t* kv_bar = bars + 0;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* st_free = bars + 4;
  uint64_t* p_full = bars + 5;
  uint64_t* dkv_done = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sm100::mbar_init(kv_bar, 1);
    sm100::mbar_init(qdo_full, 1);
    sm100::mbar_init(qdo_empty, 1);
    sm100::mbar_init(s_full, 1);
    sm100::mbar_init(st_free, 128);
    sm100::mbar_init(p_full, 128);
    sm100::mbar_init(dkv_done, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_S = tmem, TM_DP = tmem + 128, TM_DV = tmem + 256, TM_DK = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      const CUtensorMap* km = mode == 0 ? &maps.k : &maps.pk;
      const CUtensorMap* vm = mode == 0 ? &maps.v : &maps.pv;
      sm100::mbar_expect_tx(kv_bar, 2 * TILE_BYTES);
      load_tile128(smem + SmemDKDV::K, km, kv_bar, hk * D, key_row0 + kb);
      load_tile128(smem + SmemDKDV::V, vm, kv_bar, hk * D, key_row0 + kb);
      for (int it = 0; it < niter; ++it) {
        const int h = hk * rep + it / nq, qt = it0 + it % nq;
        if (!sm100::mbar_wait(qdo_empty, (it & 1) ^ 1, err, 21)) break;
        sm100::mbar_expect_tx(qdo_full, 2 * TILE_BYTES);
        load_tile128(smem + SmemDKDV::Q, &maps.q, qdo_full, h * D, q0 + qt * BQ);
        load_tile128(smem + SmemDKDV::DO, &maps.dout, qdo_full, h * D, q0 + qt * BQ);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_SS = sm100::umma_idesc_bf16(BKV, BQ, false, false);  // S^T, dP^T
      constexpr uint32_t ID_ACC = sm100::umma_idesc_bf16(BKV, D, false, true);   // dV, dK (B MN-major)
      const uint32_t k_b = sm100::smem_addr(smem + SmemDKDV::K), v_b = sm100::smem_addr(smem + SmemDKDV::V);
      const uint32_t q_b = sm100::smem_addr(smem + SmemDKDV::Q), o_b = sm100::smem_addr(smem + SmemDKDV::DO);
      const uint32_t pt_b = sm100::smem_addr(smem + SmemDKDV::PT), ds_b = sm100::smem_addr(smem + SmemDKDV::DST);
      bool ok = sm100::mbar_wait(kv_bar, 0, err, 22);
      for (int it = 0; it < niter && ok; ++it) {
        if (!sm100::mbar_wait(qdo_full, it & 1, err, 23) || !sm100::mbar_wait(st_free, (it & 1) ^ 1, err, 24)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          sm100::umma_bf16(TM_S, kmajor_desc(k_b, kk), kmajor_desc(q_b, kk), ID_SS, kk > 0);
          sm100::umma_bf16(TM_DP, kmajor_desc(v_b, kk), kmajor_desc(o_b, kk), ID_SS, kk > 0);
        }
        sm100::umma_commit(s_full);
        if (!sm100::mbar_wait(p_full, it & 1, err, 25)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          sm100::umma_bf16(TM_DV, kmajor_desc(pt_b, kk), vmajor_desc(o_b, kk), ID_ACC, it > 0 || kk > 0);
          sm100::umma_bf16(TM_DK, kmajor_desc(ds_b, kk), vmajor_desc(q_b, kk), ID_ACC, it > 0 || kk > 0);
        }
        sm100::umma_commit(qdo_empty);
      }
      if (ok) sm100::umma_commit(dkv_done);
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane, key = kb + row;
    const bool key_ok = key < key_len;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int t = threadIdx.x - 64;  // 0..127 among the softmax threads
    const float LOG2E = 1.4426950408889634f;
    bool ok = true;
    for (int it = 0; it < niter && ok; ++it) {
      const int h = hk * rep + it / nq, qbase = (it0 + it % nq) * BQ;
      {
        const int q = qbase + t;
        const bool v = q < n;
        lse_s[t] = v ? lse[(size_t)h * T + q0 + q] * LOG2E : INFINITY;
        del_s[t] = v ? delta[(size_t)h * T + q0 + q] : 0.f;
      }
      named_sync_softmax();
      bool g = sm100::mbar_wait(s_full, it & 1, err, 26);
      if (g && it > 0) g = sm100::mbar_wait(qdo_empty, (it - 1) & 1, err, 27);  // P^T / dS^T smem free
      if (!named_and_softmax(g)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BQ / 32; ++c) {
        uint32_t rs[32], rd[32];
        sm100::tmem_ld32(TM_S + lane_off + c * 32, rs);
        sm100::tmem_ld32(TM_DP + lane_off + c * 32, rd);
        sm100::tmem_ld_wait();
        float p[32], ds[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int qq = qbase + c * 32 + e;
          const bool vis = key_ok && (mode == 1 || key <= qq);  // invalid q rows carry lse=+inf -> p=0
          const float arg = __uint_as_float(rs[e]) * scale_log2 - lse_s[c * 32 + e];
          const float pe = vis ? exp2f(arg) : 0.f;
          p[e] = pe;
          ds[e] = pe * (__uint_as_float(rd[e]) - del_s[c * 32 + e]);
        }
        store_row32_sw128(smem + SmemDKDV::PT, row, c, p);
        store_row32_sw128(smem + SmemDKDV::DST, row, c, ds);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(st_free);
      sm100::fence_proxy_async_smem();
      sm100::mbar_arrive(p_full);
      named_sync_softmax();  // lse_s / del_s are rewritten by the next iteration
    }
    const bool g = ok && sm100::mbar_wait(dkv_done, 0, err, 28);
    if (__all_sync(0xffffffffu, g)) {
      sm100::tc_fence_after();
      const size_t kstride = (size_t)Hk * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t rk[32], rv[32];
        sm100::tmem_ld32(TM_DK + lane_off + c * 32, rk);
        sm100::tmem_ld32(TM_DV + lane_off + c * 32, rv);
        sm100::tmem_ld_wait();
        if (!key_ok) continue;
        if (mode == 0) {
          __nv_bfloat16* kd = dk + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32;
          __nv_bfloat16* vd = dv + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            reinterpret_cast<__nv_bfloat162*>(kd)[e] =
                __floats2bfloat162_rn(__uint_as_float(rk[2 * e]) * scale, __uint_as_float(rk[2 * e + 1]) * scale);
            reinterpret_cast<__nv_bfloat162*>(vd)[e] =
                __floats2bfloat162_rn(__uint_as_float(rv[2 * e]), __uint_as_float(rv[2 * e + 1]));
          }
        } else {
          float4* kd = reinterpret_cast<float4*>(dpk_acc + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32);
          float4* vd = reinterpret_cast<float4*>(dpv_acc + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            atomicAdd(kd + e, make_float4(__uint_as_float(rk[4 * e]) * scale, __uint_as_float(rk[4 * e + 1]) * scale,
                                          __uint_as_float(rk[4 * e + 2]) * scale, __uint_as_float(rk[4 * e + 3]) * scale));
            atomicAdd(vd + e, make_float4(__uint_as_float(rv[4 * e]), __uint_as_float(rv[4 * e + 1]),
                                          __uint_as_float(rv[4 * e + 2]), __uint_as_float(rv[4 * e + 3])));
          }
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// Pipelined dK/dV (default): the same math as tree_attn_dkdv_sm100_kernel in 64-row query steps with
// every per-step buffer doubled -- Q/dO tiles (TMA), S^T/dP^T (TMEM) and P^T/dS^T (smem) -- so the
// TMA of step i+1 and the S^T/dP^T MMAs of step i+1 run while the softmax warps work on step i, and
// the MMA warp issues S^T(i+1) before dV/dK(i).  Shared memory: K, V 64 KB + 2 x (Q, dO) 64 KB +
// 2 x (P^T, dS^T) 64 KB; TMEM: 2 x (S^T 64 | dP^T 64) + dV 128 + dK 128 = 512 columns.
constexpr int BQ2 = 64;
constexpr int QT_BYTES = BQ2 * D * 2;   // 16 KB: two 64-column blocks of 64 rows
constexpr int PT_BYTES = BKV * BQ2 * 2; // 16 KB: one 64-column block of 128 rows

struct SmemDKDV2 {
  static constexpr int K = 0;
  static constexpr int V = K + TILE_BYTES;
  static constexpr int Q0 = V + TILE_BYTES;
  static constexpr int DO0 = Q0 + 2 * QT_BYTES;
  static constexpr int PT0 = DO0 + 2 * QT_BYTES;
  static constexpr int DS0 = PT0 + 2 * PT_BYTES;
  static constexpr int LSE = DS0 + 2 * PT_BYTES;   // [2][64] floats
  static constexpr int DEL = LSE + 512;            // [2][64] floats
  static constexpr int BAR = DEL + 512;
  static constexpr int TOTAL = BAR + 256;
};

__device__ __forceinline__ uint64_t kmajor64_desc(uint32_t base, int kk) {   // [64 rows x 128], 8 KB blocks
  return sm100::umma_desc_sw128(base + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t vmajor64_desc(uint32_t base, int kk) {   // MN-major [64 (K) x 128 (N)]
  return sm100::umma_desc_sw128(base + kk * 2048, 8192, 1024);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    tree_attn_dkdv2_sm100_kernel(const __grid_constant__ BwdMaps maps, const int* __restrict__ cu,
                                 const int* __restrict__ poff, const int* __restrict__ plen,
                                 const float* __restrict__ lse, const float* __restrict__ delta,
                                 __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv,
                                 float* __restrict__ dpk_acc, float* __restrict__ dpv_acc, int B, int T, int Hq,
                                 int Hk, float scale_log2, float scale, int* err) {
  const int mode = blockIdx.y / B, b = blockIdx.y % B, hk = blockIdx.z, rep = Hq / Hk;
  const int q0 = cu[b], n = cu[b + 1] - q0;
  const int key_len = mode == 0 ? n : plen[b];
  const int key_row0 = mode == 0 ? q0 : poff[b];
  const int kb = blockIdx.x * BKV;
  if (kb >= key_len || n <= 0) return;
  const int it0 = mode == 0 ? kb / BQ2 : 0;
  const int nq = (n + BQ2 - 1) / BQ2 - it0;
  const int niter = rep * nq;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* lse_s = reinterpret_cast<float*>(smem + SmemDKDV2::LSE);
  float* del_s = reinterpret_cast<float*>(smem + SmemDKDV2::DEL);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemDKDV2::BAR);
  uint64_t* kv_bar = bars + 0;
  uint64_t* qdo_full = bars + 1;    // [2]
  uint64_t* qdo_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;      // [2]
  uint64_t* st_free = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;      // [2]
  uint64_t* dkv_done = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sm100::mbar_init(kv_bar, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&qdo_full[i], 1);
      sm100::mbar_init(&qdo_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&st_free[i], 128);
      sm100::mbar_init(&p_full[i], 128);
    }
    sm100::mbar_init(dkv_done, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_DV = tmem + 256, TM_DK = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      const CUtensorMap* km = mode == 0 ? &maps.k : &maps.pk;
      const CUtensorMap* vm = mode == 0 ? &maps.v : &maps.pv;
      sm100::mbar_expect_tx(kv_bar, 2 * TILE_BYTES);
      load_tile128(smem + SmemDKDV2::K, km, kv_bar, hk * D, key_row0 + kb);
      load_tile128(smem + SmemDKDV2::V, vm, kv_bar, hk * D, key_row0 + kb);
      for (int it = 0; it < niter; ++it) {
        const int bi = it & 1;
        const int h = hk * rep + it / nq, qt = it0 + it % nq;
        if (!sm100::mbar_wait(&qdo_empty[bi], ((it >> 1) & 1) ^ 1, err, 41)) break;
        sm100::mbar_expect_tx(&qdo_full[bi], 2 * QT_BYTES);
        unsigned char* qd = smem + SmemDKDV2::Q0 + bi * QT_BYTES;
        unsigned char* od = smem + SmemDKDV2::DO0 + bi * QT_BYTES;
        const int row0 = q0 + qt * BQ2;
        sm100::tma_load_2d(qd, &maps.q64, &qdo_full[bi], h * D, row0);
        sm100::tma_load_2d(qd + 8192, &maps.q64, &qdo_full[bi], h * D + 64, row0);
        sm100::tma_load_2d(od, &maps.dout64, &qdo_full[bi], h * D, row0);
        sm100::tma_load_2d(od + 8192, &maps.dout64, &qdo_full[bi], h * D + 64, row0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = sm100::umma_idesc_bf16(BKV, BQ2, false, false);   // S^T, dP^T: 128 x 64
      constexpr uint32_t ID_ACC = sm100::umma_idesc_bf16(BKV, D, false, true);    // dV, dK: 128 x 128
      const uint32_t k_b = sm100::smem_addr(smem + SmemDKDV2::K), v_b = sm100::smem_addr(smem + SmemDKDV2::V);
      bool ok = sm100::mbar_wait(kv_bar, 0, err, 42);
      auto issue_s = [&](int j) -> bool {
        const int bj = j & 1;
        if (!sm100::mbar_wait(&qdo_full[bj], (j >> 1) & 1, err, 43)) return false;
        if (!sm100::mbar_wait(&st_free[bj], ((j >> 1) & 1) ^ 1, err, 44)) return false;
        sm100::tc_fence_after();
        const uint32_t q_b = sm100::smem_addr(smem + SmemDKDV2::Q0 + bj * QT_BYTES);
        const uint32_t o_b = sm100::smem_addr(smem + SmemDKDV2::DO0 + bj * QT_BYTES);
        const uint32_t tm_s = tmem + bj * 128, tm_dp = tmem + bj * 128 + 64;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          sm100::umma_bf16(tm_s, kmajor_desc(k_b, kk), kmajor64_desc(q_b, kk), ID_S, kk > 0);
          sm100::umma_bf16(tm_dp, kmajor_desc(v_b, kk), kmajor64_desc(o_b, kk), ID_S, kk > 0);
        }
        sm100::umma_commit(&s_full[bj]);
        return true;
      };
      if (ok && niter > 0) ok = issue_s(0);
      for (int it = 0; it < niter && ok; ++it) {
        if (it + 1 < niter && !issue_s(it + 1)) {
          ok = false;
          break;
        }
        const int bi = it & 1;
        if (!sm100::mbar_wait(&p_full[bi], (it >> 1) & 1, err, 45)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t q_b = sm100::smem_addr(smem + SmemDKDV2::Q0 + bi * QT_BYTES);
        const uint32_t o_b = sm100::smem_addr(smem + SmemDKDV2::DO0 + bi * QT_BYTES);
        const uint32_t pt_b = sm100::smem_addr(smem + SmemDKDV2::PT0 + bi * PT_BYTES);
        const uint32_t ds_b = sm100::smem_addr(smem + SmemDKDV2::DS0 + bi * PT_BYTES);
#pragma unroll
        for (int kk = 0; kk < BQ2 / 16; ++kk) {
          sm100::umma_bf16(TM_DV, kmajor_desc(pt_b, kk), vmajor64_desc(o_b, kk), ID_ACC, it > 0 || kk > 0);
          sm100::umma_bf16(TM_DK, kmajor_desc(ds_b, kk), vmajor64_desc(q_b, kk), ID_ACC, it > 0 || kk > 0);
        }
        sm100::umma_commit(&qdo_empty[bi]);
      }
      if (ok) sm100::umma_commit(dkv_done);
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane, key = kb + row;
    const bool key_ok = key < key_len;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int t = threadIdx.x - 64;  // 0..127 among the softmax threads
    const float LOG2E = 1.4426950408889634f;
    bool ok = true;
    for (int it = 0; it < niter && ok; ++it) {
      const int bi = it & 1;
      const int h = hk * rep + it / nq, qbase = (it0 + it % nq) * BQ2;
      if (t < BQ2) {
        const int q = qbase + t;
        const bool v = q < n;
        lse_s[bi * 64 + t] = v ? lse[(size_t)h * T + q0 + q] * LOG2E : INFINITY;
        del_s[bi * 64 + t] = v ? delta[(size_t)h * T + q0 + q] : 0.f;
      }
      named_sync_softmax();
      bool g = sm100::mbar_wait(&s_full[bi], (it >> 1) & 1, err, 46);
      if (g && it >= 2) g = sm100::mbar_wait(&qdo_empty[bi], ((it >> 1) & 1) ^ 1, err, 47);  // P^T/dS^T[bi] free
      if (!named_and_softmax(g)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const uint32_t tm_s = tmem + bi * 128, tm_dp = tmem + bi * 128 + 64;
      unsigned char* pt = smem + SmemDKDV2::PT0 + bi * PT_BYTES;
      unsigned char* dst = smem + SmemDKDV2::DS0 + bi * PT_BYTES;
      // S^T and dP^T of the 64 queries in flight together, one wait
      uint32_t rs0[32], rd0[32], rs1[32], rd1[32];
      sm100::tmem_ld32(tm_s + lane_off, rs0);
      sm100::tmem_ld32(tm_dp + lane_off, rd0);
      sm100::tmem_ld32(tm_s + lane_off + 32, rs1);
      sm100::tmem_ld32(tm_dp + lane_off + 32, rd1);
      sm100::tmem_ld_wait();
      sm100::tmem_regs_ready(rs0);
      sm100::tmem_regs_ready(rd0);
      sm100::tmem_regs_ready(rs1);
      sm100::tmem_regs_ready(rd1);
      // prefix keys, and own keys below every query of the step, need no causal test (invalid query
      // rows carry lse = +inf, so their p is 0 either way)
      const bool all_vis = mode == 1 || kb + BKV - 1 <= qbase;
      const float* lse_b = lse_s + bi * 64;
      const float* del_b = del_s + bi * 64;
#pragma unroll
      for (int c = 0; c < BQ2 / 32; ++c) {
        float p[32], ds[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float sv = __uint_as_float(c == 0 ? rs0[e] : rs1[e]);
          const float dpv = __uint_as_float(c == 0 ? rd0[e] : rd1[e]);
          const bool vis = key_ok && (all_vis || key <= qbase + c * 32 + e);
          const float pe = vis ? exp2f(fmaf(sv, scale_log2, -lse_b[c * 32 + e])) : 0.f;
          p[e] = pe;
          ds[e] = pe * (dpv - del_b[c * 32 + e]);
        }
        store_row32_sw128(pt, row, c, p);
        store_row32_sw128(dst, row, c, ds);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&st_free[bi]);
      sm100::fence_proxy_async_smem();
      sm100::mbar_arrive(&p_full[bi]);
    }
    const bool g = ok && sm100::mbar_wait(dkv_done, 0, err, 48);
    if (__all_sync(0xffffffffu, g)) {
      sm100::tc_fence_after();
      const size_t kstride = (size_t)Hk * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t rk[32], rv[32];
        sm100::tmem_ld32(TM_DK + lane_off + c * 32, rk);
        sm100::tmem_ld32(TM_DV + lane_off + c * 32, rv);
        sm100::tmem_ld_wait();
        if (!key_ok) continue;
        if (mode == 0) {
          __nv_bfloat16* kd = dk + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32;
          __nv_bfloat16* vd = dv + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            reinterpret_cast<__nv_bfloat162*>(kd)[e] =
                __floats2bfloat162_rn(__uint_as_float(rk[2 * e]) * scale, __uint_as_float(rk[2 * e + 1]) * scale);
            reinterpret_cast<__nv_bfloat162*>(vd)[e] =
                __floats2bfloat162_rn(__uint_as_float(rv[2 * e]), __uint_as_float(rv[2 * e + 1]));
          }
        } else {
          float4* kd = reinterpret_cast<float4*>(dpk_acc + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32);
          float4* vd = reinterpret_cast<float4*>(dpv_acc + (size_t)(key_row0 + key) * kstride + (size_t)hk * D + c * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            atomicAdd(kd + e, make_float4(__uint_as_float(rk[4 * e]) * scale, __uint_as_float(rk[4 * e + 1]) * scale,
                                          __uint_as_float(rk[4 * e + 2]) * scale, __uint_as_float(rk[4 * e + 3]) * scale));
            atomicAdd(vd + e, make_float4(__uint_as_float(rv[4 * e]), __uint_as_float(rv[4 * e + 1]),
                                          __uint_as_float(rv[4 * e + 2]), __uint_as_float(rv[4 * e + 3])));
          }
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

struct SmemDQ {
  static constexpr int Q = 0;
  static constexpr int DO = Q + TILE_BYTES;
  static constexpr int K0 = DO + TILE_BYTES;              // 2 stages of K
  static constexpr int V0 = K0 + 2 * TILE_BYTES;          // 2 stages of V
  static constexpr int DS = V0 + 2 * TILE_BYTES;
  static constexpr int BAR = DS + TILE_BYTES;
  static constexpr int TOTAL = BAR + 256;
};

__global__ void __launch_bounds__(NUM_THREADS, 1)
    tree_attn_dq_sm100_kernel(const __grid_constant__ BwdMaps maps, const int* __restrict__ cu,
                              const int* __restrict__ poff, const int* __restrict__ plen,
                              const float* __restrict__ lse, const float* __restrict__ delta,
                              __nv_bfloat16* __restrict__ dq, int T, int Hq, int Hk, float scale_log2, float scale,
                              int* err) {
  const int seq = blockIdx.y, h = blockIdx.z, hk = h / (Hq / Hk);
  const int q0 = cu[seq], n = cu[seq + 1] - q0;
  const int m0 = blockIdx.x * BQ;
  if (m0 >= n) return;
  const int po = poff[seq], pl = plen[seq];
  const int n_pre = (pl + BKV - 1) / BKV;
  const int n_self = (min(n, m0 + BQ) + BKV - 1) / BKV;
  const int ntiles = n_pre + n_self;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemDQ::BAR);
  uint64_t* qdo_bar = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* sd_free = bars + 6;
  uint64_t* ds_full = bars + 7;
  uint64_t* ds_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sm100::mbar_init(qdo_bar, 1);
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&kv_full[i], 1);
      sm100::mbar_init(&kv_empty[i], 1);
    }
    sm100::mbar_init(s_full, 1);
    sm100::mbar_init(sd_free, 128);
    sm100::mbar_init(ds_full, 128);
    sm100::mbar_init(ds_done, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_S = tmem, TM_DP = tmem + 128, TM_DQ = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      sm100::mbar_expect_tx(qdo_bar, 2 * TILE_BYTES);
      load_tile128(smem + SmemDQ::Q, &maps.q, qdo_bar, h * D, q0 + m0);
      load_tile128(smem + SmemDQ::DO, &maps.dout, qdo_bar, h * D, q0 + m0);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        if (!sm100::mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, err, 31)) break;
        sm100::mbar_expect_tx(&kv_full[st], 2 * TILE_BYTES);
        const bool pre = j < n_pre;
        const int r0 = pre ? po + j * BKV : q0 + (j - n_pre) * BKV;
        load_tile128(smem + SmemDQ::K0 + st * TILE_BYTES, pre ? &maps.pk : &maps.k, &kv_full[st], hk * D, r0);
        load_tile128(smem + SmemDQ::V0 + st * TILE_BYTES, pre ? &maps.pv : &maps.v, &kv_full[st], hk * D, r0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_SS = sm100::umma_idesc_bf16(BQ, BKV, false, false);
      constexpr uint32_t ID_DQ = sm100::umma_idesc_bf16(BQ, D, false, true);
      const uint32_t q_b = sm100::smem_addr(smem + SmemDQ::Q), o_b = sm100::smem_addr(smem + SmemDQ::DO);
      const uint32_t ds_b = sm100::smem_addr(smem + SmemDQ::DS);
      bool ok = sm100::mbar_wait(qdo_bar, 0, err, 32);
      for (int j = 0; j < ntiles && ok; ++j) {
        const int st = j & 1;
        if (!sm100::mbar_wait(&kv_full[st], (j >> 1) & 1, err, 33) || !sm100::mbar_wait(sd_free, (j & 1) ^ 1, err, 34)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t k_b = sm100::smem_addr(smem + SmemDQ::K0 + st * TILE_BYTES);
        const uint32_t v_b = sm100::smem_addr(smem + SmemDQ::V0 + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          sm100::umma_bf16(TM_S, kmajor_desc(q_b, kk), kmajor_desc(k_b, kk), ID_SS, kk > 0);
          sm100::umma_bf16(TM_DP, kmajor_desc(o_b, kk), kmajor_desc(v_b, kk), ID_SS, kk > 0);
        }
        sm100::umma_commit(s_full);
        if (!sm100::mbar_wait(ds_full, j & 1, err, 35)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          sm100::umma_bf16(TM_DQ, kmajor_desc(ds_b, kk), vmajor_desc(k_b, kk), ID_DQ, j > 0 || kk > 0);
        sm100::umma_commit(&kv_empty[st]);
        sm100::umma_commit(ds_done);
      }
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane, qi = m0 + row;
    const bool row_ok = qi < n;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float LOG2E = 1.4426950408889634f;
    const float lse_r = row_ok ? lse[(size_t)h * T + q0 + qi] * LOG2E : 0.f;
    const float del_r = row_ok ? delta[(size_t)h * T + q0 + qi] : 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      bool g = sm100::mbar_wait(s_full, j & 1, err, 36);
      if (g && j > 0) g = sm100::mbar_wait(ds_done, (j - 1) & 1, err, 37);
      if (!__all_sync(0xffffffffu, g)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const bool pre = j < n_pre;
      const int kbase = pre ? j * BKV : (j - n_pre) * BKV;
      const int klim = pre ? pl : min(n, qi + 1);
#pragma unroll 1
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t rs[32], rd[32];
        sm100::tmem_ld32(TM_S + lane_off + c * 32, rs);
        sm100::tmem_ld32(TM_DP + lane_off + c * 32, rd);
        sm100::tmem_ld_wait();
        float ds[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const bool vis = row_ok && (kbase + c * 32 + e) < klim;
          const float arg = __uint_as_float(rs[e]) * scale_log2 - lse_r;
          const float pe = vis ? exp2f(arg) : 0.f;
          ds[e] = pe * (__uint_as_float(rd[e]) - del_r);
        }
        store_row32_sw128(smem + SmemDQ::DS, row, c, ds);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(sd_free);
      sm100::fence_proxy_async_smem();
      sm100::mbar_arrive(ds_full);
    }
    const bool g = ok && sm100::mbar_wait(ds_done, (ntiles - 1) & 1, err, 38);
    if (__all_sync(0xffffffffu, g)) {
      sm100::tc_fence_after();
      __nv_bfloat16* dst = dq + (size_t)(q0 + qi) * Hq * D + (size_t)h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(TM_DQ + lane_off + c * 32, r);
        sm100::tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            reinterpret_cast<__nv_bfloat162*>(dst + c * 32)[e] =
                __floats2bfloat162_rn(__uint_as_float(r[2 * e]) * scale, __uint_as_float(r[2 * e + 1]) * scale);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// Pipelined dQ (default): 64-key tiles with a three-stage K/V ring and every per-tile buffer doubled --
// S / dP in TMEM (2 x (64 | 64) columns) and dS in shared memory (2 x 16 KB) -- so the MMA warp issues
// S(j+1), dP(j+1) before dQ += dS(j) K(j) and the tensor pipe works while the softmax warps form dS(j).
// Eight softmax warps (each TMEM lane quarter served twice, one 32-key half each) keep the exp / dS
// work of a tile shorter than its MMAs.
// Shared memory: Q, dO 64 KB + 3 x (K, V) 96 KB + 2 x dS 32 KB; TMEM: 256 (S, dP) + 128 (dQ) columns.
constexpr int BKV2 = 64;
constexpr int KT_BYTES = BKV2 * D * 2;   // 16 KB: two 64-column blocks of 64 rows
constexpr int DS2_BYTES = BQ * BKV2 * 2; // 16 KB: one 64-column block of 128 rows
constexpr int DQ_STAGES = 3;
constexpr int DQ2_THREADS = 320;  // TMA warp, MMA warp, 8 softmax warps (two per TMEM lane quarter)

struct SmemDQ2 {
  static constexpr int Q = 0;
  static constexpr int DO = Q + TILE_BYTES;
  static constexpr int K0 = DO + TILE_BYTES;
  static constexpr int V0 = K0 + DQ_STAGES * KT_BYTES;
  static constexpr int DS0 = V0 + DQ_STAGES * KT_BYTES;
  static constexpr int BAR = DS0 + 2 * DS2_BYTES;
  static constexpr int TOTAL = BAR + 256;
};

__global__ void __launch_bounds__(DQ2_THREADS, 1)
    tree_attn_dq2_sm100_kernel(const __grid_constant__ BwdMaps maps, const int* __restrict__ cu,
                               const int* __restrict__ poff, const int* __restrict__ plen,
                               const float* __restrict__ lse, const float* __restrict__ delta,
                               __nv_bfloat16* __restrict__ dq, int T, int Hq, int Hk, float scale_log2, float scale,
                               int* err) {
  const int seq = blockIdx.y, h = blockIdx.z, hk = h / (Hq / Hk);
  const int q0 = cu[seq], n = cu[seq + 1] - q0;
  const int m0 = blockIdx.x * BQ;
  if (m0 >= n) return;
  const int po = poff[seq], pl = plen[seq];
  const int n_pre = (pl + BKV2 - 1) / BKV2;
  const int n_self = (min(n, m0 + BQ) + BKV2 - 1) / BKV2;
  const int ntiles = n_pre + n_self;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemDQ2::BAR);
  uint64_t* qdo_bar = bars + 0;
  uint64_t* kv_full = bars + 1;    // [3]
  uint64_t* kv_empty = bars + 4;   // [3]
  uint64_t* s_full = bars + 7;     // [2] S, dP of a tile landed in TMEM
  uint64_t* sd_free = bars + 9;    // [2] softmax warps read S, dP of the buffer
  uint64_t* ds_full = bars + 11;   // [2] dS of the buffer written to smem
  uint64_t* ds_done = bars + 13;   // [2] dQ MMA of the buffer completed (dS smem reusable)
  uint64_t* dq_done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sm100::mbar_init(qdo_bar, 1);
    for (int i = 0; i < DQ_STAGES; ++i) {
      sm100::mbar_init(&kv_full[i], 1);
      sm100::mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&sd_free[i], 256);
      sm100::mbar_init(&ds_full[i], 256);
      sm100::mbar_init(&ds_done[i], 1);
    }
    sm100::mbar_init(dq_done, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_DQ = tmem + 256;  // S(b) at tmem + 64 b, dP(b) at tmem + 128 + 64 b

  if (warp == 0) {
    if (lane == 0) {
      sm100::mbar_expect_tx(qdo_bar, 2 * TILE_BYTES);
      load_tile128(smem + SmemDQ2::Q, &maps.q, qdo_bar, h * D, q0 + m0);
      load_tile128(smem + SmemDQ2::DO, &maps.dout, qdo_bar, h * D, q0 + m0);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % DQ_STAGES;
        if (!sm100::mbar_wait(&kv_empty[st], ((j / DQ_STAGES) & 1) ^ 1, err, 51)) break;
        sm100::mbar_expect_tx(&kv_full[st], 2 * KT_BYTES);
        const bool pre = j < n_pre;
        const int r0 = pre ? po + j * BKV2 : q0 + (j - n_pre) * BKV2;
        const CUtensorMap* km = pre ? &maps.pk64 : &maps.k64;
        const CUtensorMap* vm = pre ? &maps.pv64 : &maps.v64;
        unsigned char* kd = smem + SmemDQ2::K0 + st * KT_BYTES;
        unsigned char* vd = smem + SmemDQ2::V0 + st * KT_BYTES;
        sm100::tma_load_2d(kd, km, &kv_full[st], hk * D, r0);
        sm100::tma_load_2d(kd + 8192, km, &kv_full[st], hk * D + 64, r0);
        sm100::tma_load_2d(vd, vm, &kv_full[st], hk * D, r0);
        sm100::tma_load_2d(vd + 8192, vm, &kv_full[st], hk * D + 64, r0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = sm100::umma_idesc_bf16(BQ, BKV2, false, false);  // S, dP: 128 x 64
      constexpr uint32_t ID_DQ = sm100::umma_idesc_bf16(BQ, D, false, true);     // dQ: 128 x 128
      const uint32_t q_b = sm100::smem_addr(smem + SmemDQ2::Q), o_b = sm100::smem_addr(smem + SmemDQ2::DO);
      auto issue_s = [&](int j) -> bool {
        const int st = j % DQ_STAGES, b = j & 1;
        if (!sm100::mbar_wait(&kv_full[st], (j / DQ_STAGES) & 1, err, 52)) return false;
        if (!sm100::mbar_wait(&sd_free[b], ((j >> 1) & 1) ^ 1, err, 53)) return false;
        sm100::tc_fence_after();
        const uint32_t k_b = sm100::smem_addr(smem + SmemDQ2::K0 + st * KT_BYTES);
        const uint32_t v_b = sm100::smem_addr(smem + SmemDQ2::V0 + st * KT_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          sm100::umma_bf16(tmem + b * 64, kmajor_desc(q_b, kk), kmajor64_desc(k_b, kk), ID_S, kk > 0);
          sm100::umma_bf16(tmem + 128 + b * 64, kmajor_desc(o_b, kk), kmajor64_desc(v_b, kk), ID_S, kk > 0);
        }
        sm100::umma_commit(&s_full[b]);
        return true;
      };
      auto issue_dq = [&](int j) -> bool {
        const int st = j % DQ_STAGES, b = j & 1;
        if (!sm100::mbar_wait(&ds_full[b], (j >> 1) & 1, err, 54)) return false;
        sm100::tc_fence_after();
        const uint32_t k_b = sm100::smem_addr(smem + SmemDQ2::K0 + st * KT_BYTES);
        const uint32_t ds_b = sm100::smem_addr(smem + SmemDQ2::DS0 + b * DS2_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV2 / 16; ++kk)
          sm100::umma_bf16(TM_DQ, kmajor_desc(ds_b, kk), vmajor64_desc(k_b, kk), ID_DQ, j > 0 || kk > 0);
        sm100::umma_commit(&kv_empty[st]);
        sm100::umma_commit(&ds_done[b]);
        return true;
      };
      bool ok = sm100::mbar_wait(qdo_bar, 0, err, 55) && issue_s(0);
      for (int j = 0; j < ntiles && ok; ++j) {
        if (j + 1 < ntiles) ok = issue_s(j + 1);
        if (ok) ok = issue_dq(j);
      }
      if (ok) sm100::umma_commit(dq_done);
    }
  } else {
    // eight softmax warps: warp w serves TMEM lanes 32 (w % 4) .. (rows) and the 32-key half (w - 2) / 4
    const int quarter = warp & 3, half = (warp - 2) >> 2, row = quarter * 32 + lane, qi = m0 + row;
    const bool row_ok = qi < n;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float LOG2E = 1.4426950408889634f;
    const float lse_r = row_ok ? lse[(size_t)h * T + q0 + qi] * LOG2E : 0.f;
    const float del_r = row_ok ? delta[(size_t)h * T + q0 + qi] : 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int b = j & 1;
      bool g = sm100::mbar_wait(&s_full[b], (j >> 1) & 1, err, 56);
      if (g && j >= 2) g = sm100::mbar_wait(&ds_done[b], ((j >> 1) & 1) ^ 1, err, 57);  // dS[b] of j-2 consumed
      if (!__all_sync(0xffffffffu, g)) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      const bool pre = j < n_pre;
      const int kbase = pre ? j * BKV2 : (j - n_pre) * BKV2;
      const int klim = pre ? pl : min(n, qi + 1);
      unsigned char* ds_tile = smem + SmemDQ2::DS0 + b * DS2_BYTES;
      {
        const int c = half;
        uint32_t rs[32], rd[32];
        sm100::tmem_ld32(tmem + b * 64 + lane_off + c * 32, rs);
        sm100::tmem_ld32(tmem + 128 + b * 64 + lane_off + c * 32, rd);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(rs);
        sm100::tmem_regs_ready(rd);
        float ds[32];
        // keys of this half wholly visible to every row of the warp: no per-key test
        const bool all_vis = __all_sync(0xffffffffu, row_ok && kbase + c * 32 + 32 <= klim);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const bool vis = all_vis || (row_ok && (kbase + c * 32 + e) < klim);
          const float pe = vis ? exp2f(fmaf(__uint_as_float(rs[e]), scale_log2, -lse_r)) : 0.f;
          ds[e] = pe * (__uint_as_float(rd[e]) - del_r);
        }
        store_row32_sw128(ds_tile, row, c, ds);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&sd_free[b]);
      sm100::fence_proxy_async_smem();
      sm100::mbar_arrive(&ds_full[b]);
    }
    const bool g = ok && sm100::mbar_wait(dq_done, 0, err, 58);
    if (__all_sync(0xffffffffu, g)) {
      sm100::tc_fence_after();
      __nv_bfloat16* dst = dq + (size_t)(q0 + qi) * Hq * D + (size_t)h * D;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        uint32_t r[32];
        sm100::tmem_ld32(TM_DQ + lane_off + c * 32, r);
        sm100::tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            reinterpret_cast<__nv_bfloat162*>(dst + c * 32)[e] =
                __floats2bfloat162_rn(__uint_as_float(r[2 * e]) * scale, __uint_as_float(r[2 * e + 1]) * scale);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// delta[h, t] = <dO[t, h, :], O[t, h, :]>: each half-warp reduces one 128-wide row (16 lanes x 16 bytes);
// a warp takes two pairs of rows per step (loop bounds uniform across the warp for the shuffles)
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                             float* __restrict__ delta, int T, int Hq) {
  const int lane = threadIdx.x & 31, sub = lane & 15, half = lane >> 4;
  const long total = (long)T * Hq;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  const long w = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (long base = 2 * w; base < total; base += 4 * nwarps) {
    const long r0 = base + half, r1 = base + 2 * nwarps + half;
    const bool v0 = r0 < total, v1 = r1 < total;
    bb::bf16x8 a0{}, o0{}, a1{}, o1{};
    if (v0) {
      a0 = reinterpret_cast<const bb::bf16x8*>(dout + r0 * D)[sub];
      o0 = reinterpret_cast<const bb::bf16x8*>(out + r0 * D)[sub];
    }
    if (v1) {
      a1 = reinterpret_cast<const bb::bf16x8*>(dout + r1 * D)[sub];
      o1 = reinterpret_cast<const bb::bf16x8*>(out + r1 * D)[sub];
    }
    float fa[8], fo[8], s0 = 0.f, s1 = 0.f;
    bb::unpack8(a0, fa);
    bb::unpack8(o0, fo);
#pragma unroll
    for (int e = 0; e < 8; ++e) s0 += fa[e] * fo[e];
    bb::unpack8(a1, fa);
    bb::unpack8(o1, fo);
#pragma unroll
    for (int e = 0; e < 8; ++e) s1 += fa[e] * fo[e];
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, off);
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    }
    if (sub == 0) {
      if (v0) delta[(size_t)(r0 % Hq) * T + r0 / Hq] = s0;
      if (v1) delta[(size_t)(r1 % Hq) * T + r1 / Hq] = s1;
    }
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16(src[i]);
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

// Row-major [rows, cols] bf16 -> map with box {64 cols, box_rows}, 128-byte swizzle.
void encode_rows(CUtensorMap* m, const void* base, long rows, long cols, int box_rows = 128) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0 && (cols * 2) % 16 == 0, "attention TMA alignment");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)std::max<long>(rows, 1)};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (attention) failed: ", (int)r);
}

AttnMaps* attn_map_storage() {
  thread_local AttnMaps* p = nullptr;
  if (!p) {
    void* raw = nullptr;
    TORCH_CHECK(posix_memalign(&raw, 64, sizeof(AttnMaps)) == 0, "posix_memalign failed");
    p = reinterpret_cast<AttnMaps*>(raw);
  }
  return p;
}

torch::Tensor& attn_error_word() {
  static torch::Tensor e;
  if (!e.defined()) e = torch::zeros({1}, torch::dtype(torch::kInt).device(torch::kCUDA));
  return e;
}

}  // namespace

std::vector<torch::Tensor> tree_attn_fwd_sm100(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor pk,
                                               torch::Tensor pv, torch::Tensor cu, torch::Tensor poff,
                                               torch::Tensor plen, int64_t max_seqlen, int64_t max_prefix,
                                               double scale) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.is_contiguous() && k.is_contiguous() &&
                  v.is_contiguous(), "q/k/v must be contiguous CUDA bf16");
  const int T = q.size(0), Hq = q.size(1), Hk = k.size(1);
  TORCH_CHECK(q.size(2) == D && k.size(2) == D, "tcgen05 attention is built for head_dim 128");
  TORCH_CHECK(Hq % Hk == 0, "GQA: Hq % Hkv");
  const int B = cu.numel() - 1;
  auto o = torch::empty_like(q);
  auto lse = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  if (T == 0 || B == 0) return {o, lse};
  at::cuda::CUDAGuard guard(q.get_device());
  {
    CUcontext cur = nullptr;
    if (cuCtxGetCurrent(&cur) != CUDA_SUCCESS || cur == nullptr) BB_CHECK_CUDA(cudaFree(nullptr));
  }
  AttnMaps* maps = attn_map_storage();
  encode_rows(&maps->q, q.data_ptr(), T, (long)Hq * D);
  encode_rows(&maps->k, k.data_ptr(), T, (long)Hk * D);
  encode_rows(&maps->v, v.data_ptr(), T, (long)Hk * D);
  const bool has_p = pk.numel() > 0;
  encode_rows(&maps->pk, has_p ? pk.data_ptr() : k.data_ptr(), has_p ? pk.size(0) : T, (long)Hk * D);
  encode_rows(&maps->pv, has_p ? pv.data_ptr() : v.data_ptr(), has_p ? pv.size(0) : T, (long)Hk * D);
  const int smem = Smem::TOTAL + 1024;
  auto kern = tree_attn_fwd_sm100_kernel;
  static unsigned long long attr_done = 0;
  bb::set_smem_attr_once(kern, smem, attr_done);
  dim3 grid((max_seqlen + BQ - 1) / BQ, B, Hq);
  const int* cup = cu.data_ptr<int>();
  const int* pop = poff.data_ptr<int>();
  const int* plp = plen.data_ptr<int>();
  __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  float* lp = lse.data_ptr<float>();
  float sl2 = (float)(scale * 1.4426950408889634);
  int* err = attn_error_word().data_ptr<int>();
  int Ti = T, Hqi = Hq, Hki = Hk;
  void* args[] = {maps, &cup, &pop, &plp, &op, &lp, &Ti, &Hqi, &Hki, &sl2, &err};
  BB_CHECK_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(kern), grid, dim3(NUM_THREADS), args, smem,
                                 at::cuda::getCurrentCUDAStream()));
  BB_POST_LAUNCH();
  return {o, lse};
}

int64_t attn_error_code() { return attn_error_word().item<int>(); }

void attn_phase_profile(bool enable) {
  const int on = enable ? 1 : 0;
  unsigned long long zero[8] = {};
  BB_CHECK_CUDA(cudaMemcpyToSymbol(g_attn_prof, zero, sizeof(zero)));
  BB_CHECK_CUDA(cudaMemcpyToSymbol(g_attn_prof_on, &on, sizeof(on)));
}

torch::Tensor attn_phase_read() {
  unsigned long long tab[8];
  BB_CHECK_CUDA(cudaMemcpyFromSymbol(tab, g_attn_prof, sizeof(tab)));
  auto out = torch::empty({8}, torch::TensorOptions().dtype(torch::kInt64));
  for (int i = 0; i < 8; ++i) out[i] = (int64_t)tab[i];
  return out;
}

std::vector<torch::Tensor> tree_attn_bwd_sm100(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                               torch::Tensor pk, torch::Tensor pv, torch::Tensor o, torch::Tensor lse,
                                               torch::Tensor cu, torch::Tensor poff, torch::Tensor plen,
                                               int64_t max_seqlen, int64_t max_prefix, double scale) {
  TORCH_CHECK(dout.is_contiguous() && q.size(2) == D, "tcgen05 attention backward: contiguous, head_dim 128");
  const int T = q.size(0), Hq = q.size(1), Hk = k.size(1);
  const int B = cu.numel() - 1;
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k), dv = torch::empty_like(v);
  const bool has_p = pk.numel() > 0;
  auto dpk = torch::zeros_like(pk), dpv = torch::zeros_like(pv);
  if (T == 0 || B == 0) return {dq, dk, dv, dpk, dpv};
  at::cuda::CUDAGuard guard(q.get_device());
  {
    CUcontext cur = nullptr;
    if (cuCtxGetCurrent(&cur) != CUDA_SUCCESS || cur == nullptr) BB_CHECK_CUDA(cudaFree(nullptr));
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  auto delta = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  {
    const int blocks = (int)std::max<long>(1, std::min<long>(((long)T * Hq + 31) / 32, 148l * 16));
    delta_kernel<<<blocks, 256, 0, stream>>>((const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)o.data_ptr(),
                                             delta.data_ptr<float>(), T, Hq);
    BB_POST_LAUNCH();
  }
  torch::Tensor dpk_acc, dpv_acc;
  if (has_p) {
    dpk_acc = torch::zeros(pk.sizes(), pk.options().dtype(at::kFloat));
    dpv_acc = torch::zeros(pv.sizes(), pv.options().dtype(at::kFloat));
  }
  static thread_local BwdMaps* maps = nullptr;
  if (!maps) {
    void* raw = nullptr;
    TORCH_CHECK(posix_memalign(&raw, 64, sizeof(BwdMaps)) == 0, "posix_memalign failed");
    maps = reinterpret_cast<BwdMaps*>(raw);
  }
  encode_rows(&maps->q, q.data_ptr(), T, (long)Hq * D);
  encode_rows(&maps->k, k.data_ptr(), T, (long)Hk * D);
  encode_rows(&maps->v, v.data_ptr(), T, (long)Hk * D);
  encode_rows(&maps->pk, has_p ? pk.data_ptr() : k.data_ptr(), has_p ? pk.size(0) : T, (long)Hk * D);
  encode_rows(&maps->pv, has_p ? pv.data_ptr() : v.data_ptr(), has_p ? pv.size(0) : T, (long)Hk * D);
  encode_rows(&maps->dout, dout.data_ptr(), T, (long)Hq * D);
  encode_rows(&maps->q64, q.data_ptr(), T, (long)Hq * D, 64);
  encode_rows(&maps->dout64, dout.data_ptr(), T, (long)Hq * D, 64);
  encode_rows(&maps->k64, k.data_ptr(), T, (long)Hk * D, 64);
  encode_rows(&maps->v64, v.data_ptr(), T, (long)Hk * D, 64);
  encode_rows(&maps->pk64, has_p ? pk.data_ptr() : k.data_ptr(), has_p ? pk.size(0) : T, (long)Hk * D, 64);
  encode_rows(&maps->pv64, has_p ? pv.data_ptr() : v.data_ptr(), has_p ? pv.size(0) : T, (long)Hk * D, 64);
  const int* cup = cu.data_ptr<int>();
  const int* pop = poff.data_ptr<int>();
  const int* plp = plen.data_ptr<int>();
  const float* lsep = lse.data_ptr<float>();
  const float* delp = delta.data_ptr<float>();
  float sl2 = (float)(scale * 1.4426950408889634), sc = (float)scale;
  int* err = attn_error_word().data_ptr<int>();
  int Bi = B, Ti = T, Hqi = Hq, Hki = Hk;
  {
    static const bool v1 = getenv("BB_ATTN_DKDV") && std::string(getenv("BB_ATTN_DKDV")) == "v1";
    auto kern = v1 ? tree_attn_dkdv_sm100_kernel : tree_attn_dkdv2_sm100_kernel;
    const int smem = (v1 ? SmemDKDV::TOTAL : SmemDKDV2::TOTAL) + 1024;
    static unsigned long long attr_done = 0;
    bb::set_smem_attr_once(kern, smem, attr_done);
    const long xt = std::max<long>((max_seqlen + BKV - 1) / BKV, has_p ? (max_prefix + BKV - 1) / BKV : 0);
    dim3 grid((unsigned)std::max<long>(xt, 1), (unsigned)(has_p ? 2 * B : B), (unsigned)Hk);
    __nv_bfloat16* dkp = (__nv_bfloat16*)dk.data_ptr();
    __nv_bfloat16* dvp = (__nv_bfloat16*)dv.data_ptr();
    float* dpkp = has_p ? dpk_acc.data_ptr<float>() : nullptr;
    float* dpvp = has_p ? dpv_acc.data_ptr<float>() : nullptr;
    void* args[] = {maps, &cup, &pop, &plp, &lsep, &delp, &dkp, &dvp, &dpkp, &dpvp, &Bi, &Ti, &Hqi, &Hki, &sl2, &sc, &err};
    BB_CHECK_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(kern), grid, dim3(NUM_THREADS), args, smem, stream));
    BB_POST_LAUNCH();
  }
  {
    static const bool dq_v1 = getenv("BB_ATTN_DQ") && std::string(getenv("BB_ATTN_DQ")) == "v1";
    auto kern = dq_v1 ? tree_attn_dq_sm100_kernel : tree_attn_dq2_sm100_kernel;
    const int smem = (dq_v1 ? SmemDQ::TOTAL : SmemDQ2::TOTAL) + 1024;
    static unsigned long long attr_done = 0;
    bb::set_smem_attr_once(kern, smem, attr_done);
    dim3 grid((unsigned)((max_seqlen + BQ - 1) / BQ), (unsigned)B, (unsigned)Hq);
    __nv_bfloat16* dqp = (__nv_bfloat16*)dq.data_ptr();
    void* args[] = {maps, &cup, &pop, &plp, &lsep, &delp, &dqp, &Ti, &Hqi, &Hki, &sl2, &sc, &err};
    BB_CHECK_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(kern), grid, dim3(dq_v1 ? NUM_THREADS : DQ2_THREADS), args,
                                   smem, stream));
    BB_POST_LAUNCH();
  }
  if (has_p) {
    const long nel = dpk.numel();
    const int blocks = (int)std::min<long>((nel + 255) / 256, 148l * 16);
    f32_to_bf16_kernel<<<blocks, 256, 0, stream>>>(dpk_acc.data_ptr<float>(), (__nv_bfloat16*)dpk.data_ptr(), nel);
    BB_POST_LAUNCH();
    f32_to_bf16_kernel<<<blocks, 256, 0, stream>>>(dpv_acc.data_ptr<float>(), (__nv_bfloat16*)dpv.data_ptr(), nel);
    BB_POST_LAUNCH();
  }
  return {dq, dk, dv, dpk, dpv};
}
