// gemm_pair.cu -- persistent CTA-pair (cta_group::2) block-scaled GEMM.
//
// C[M,N] = alpha * A[M,K] . B[N,K]^T for NVFP4 (kind::mxf4nvf4.block16) and
// MXFP8 (kind::mxf8f6f4.block_scale), the B200 replacement for the
// reference's NVFP4 GEMM backends (CUTLASS example 72b,
// GEMMquant_sm110/build_and_run.sh:38-75; the disabled 2-SM tc6 kernel,
// GEMMsm110/include/backends/tc6_nvfp4.cuh:86-332).
//
// A cluster of two CTAs (one per SM) owns a 256 x 256 output tile.  Each CTA
// loads its own 128 rows of A and its own 128-row half of B; the leader CTA
// (rank 0) issues tcgen05.mma.cta_group::2 (M = 256, N = 256), which reads A
// and B from both CTAs' shared memory and accumulates rows [0,128) in the
// leader's TMEM and rows [128,256) in the peer's.
//
// Scale factors reach TMEM through tcgen05.st from registers, not through
// tcgen05.cp: copy instructions execute in the tensor pipe in order with the
// MMAs and cost a roughly fixed time each (12 per stage for NVFP4), which
// measured as ~45% of the kernel.  Four stager warps per CTA -- one per
// 32-lane TMEM quadrant -- read each stage's 512-byte scale chunks from shared
// memory and write the layout the MMA reads (row r at lane r%32 of every
// quadrant, column r/32, byte = scale index) for their own quadrant.
//
// Roles (both CTAs, 10 warps):
//   warp 0      TMA producer.  A/B loads complete on the LEADER's full barrier
//               (cta_group::2 form, armed by the leader with both CTAs'
//               bytes); scale loads complete on this CTA's own sf_full barrier.
//   warp 1      TMEM allocation for the pair; in the leader, the MMA issuer.
//   warps 2..5  epilogue: each CTA drains its own accumulator rows.
//   warps 6..9  scale stagers.
// No TMA load uses cluster multicast.  Every wait is bounded (qg_ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

template <bool kFp4>
struct PairCfg {
  static constexpr int kBM = 128;       // rows of A per CTA (256 per pair)
  static constexpr int kBN = 256;       // N of the pair tile
  static constexpr int kBNHalf = 128;   // rows of B each CTA loads
  static constexpr int kBKBytes = 128;  // K bytes per stage (one SWIZZLE_128B row)
  static constexpr int kStages = kFp4 ? 5 : 6;
  static constexpr int kMmaPerStage = 4;
  static constexpr int kSfChunks = kFp4 ? 4 : 1;  // 512-B chunks along K per 128 rows
  static constexpr int kABytes = kBM * kBKBytes;
  static constexpr int kBBytes = kBNHalf * kBKBytes;
  static constexpr int kSfaBytes = kSfChunks * 512;
  static constexpr int kSfbBytes = kSfChunks * 512 * 2;  // all 256 N rows in each CTA
  static constexpr int kAbTx = kABytes + kBBytes;
  static constexpr int kSfTx = kSfaBytes + kSfbBytes;
  static constexpr int kStageBytes = (kAbTx + kSfTx + 1023) / 1024 * 1024;
  static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
  static constexpr int kSfaCols = kSfChunks * 4;
  static constexpr int kSfbCols = kSfChunks * 8;
  static constexpr int kTmemSfBase = kBN;
  static constexpr int kTmemSfStageCols = kSfaCols + kSfbCols;
  static constexpr int kTmemCols = 512;
  static_assert(kTmemSfBase + kStages * kTmemSfStageCols <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr int kThreads = 320;
};

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void spin_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) {
  }
}

// One stage's scales of this warp's TMEM quadrant: SFA chunks (4 columns
// each, the 16-byte row r of a chunk holds rows r, r+32, r+64, r+96) and the
// two 128-row SFB blocks per chunk (8 columns per chunk).
template <bool kFp4>
__device__ __forceinline__ void stage_scales(const uint8_t* ssfa, const uint8_t* ssfb,
                                             uint32_t t_quad, uint32_t sfa_col, uint32_t sfb_col,
                                             int lane) {
  using Cfg = PairCfg<kFp4>;
  uint32_t a[Cfg::kSfaCols];
  uint32_t b[Cfg::kSfbCols];
#pragma unroll
  for (int c = 0; c < Cfg::kSfChunks; ++c) {
    const uint4 v = lds128(ssfa + c * 512 + lane * 16);
    a[4 * c] = v.x;
    a[4 * c + 1] = v.y;
    a[4 * c + 2] = v.z;
    a[4 * c + 3] = v.w;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 w = lds128(ssfb + (c * 2 + h) * 512 + lane * 16);
      b[8 * c + 4 * h] = w.x;
      b[8 * c + 4 * h + 1] = w.y;
      b[8 * c + 4 * h + 2] = w.z;
      b[8 * c + 4 * h + 3] = w.w;
    }
  }
  tmem_st_32x32b<Cfg::kSfaCols>(t_quad + sfa_col, a);
  tmem_st_32x32b<Cfg::kSfbCols>(t_quad + sfb_col, b);
}

template <bool kFp4, bool kOutBf16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = PairCfg<kFp4>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;                        // leader: A/B bytes of both CTAs
  uint64_t* sf_full = bars + Cfg::kStages;          // each CTA: its scale bytes
  uint64_t* sf_ready = bars + 2 * Cfg::kStages;     // leader: 8 stager warps
  uint64_t* empty_bar = bars + 3 * Cfg::kStages;    // each CTA
  uint64_t* acc_full = bars + 4 * Cfg::kStages;     // each CTA
  uint64_t* acc_empty = acc_full + 1;               // leader: 8 epilogue warps
  uint64_t* drain_bar = acc_full + 2;               // leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 3);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int npairs = static_cast<int>(nclusters_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&sf_full[s], 1);
      mbar_init(&sf_ready[s], 8);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    fence_barrier_init();
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
    tma_prefetch_desc(&p.tm_sfa);
    tma_prefetch_desc(&p.tm_sfb);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barrier inits and TMEM allocation visible to both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  const int nkb = p.num_k_blocks;
  const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / npairs + 1 : 0;
  const int total_kb = my_tiles * nkb;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int g = 0; g < total_kb; ++g) {
        const int stage = g % Cfg::kStages;
        const uint32_t phase = static_cast<uint32_t>((g / Cfg::kStages) & 1);
        const int tile = pair + (g / nkb) * npairs;
        const int kb = g % nkb;
        const int mt = tile % p.num_m_tiles;
        const int nt = tile / p.num_m_tiles;
        if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * Cfg::kStageBytes;
        uint8_t* sb = sa + Cfg::kABytes;
        uint8_t* ssfa = sb + Cfg::kBBytes;
        uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
        const bool cp_mode = (p.diag & 16u) != 0 || (p.diag & 64u) != 0;
        if (p.diag & 4u) {
          if (leader) mbar_arrive(&full_bar[stage]);
          if (!cp_mode) mbar_arrive(&sf_full[stage]);
          continue;
        }
        if (cp_mode) {
          // Scales through tcgen05.cp issued by the MMA thread: all bytes on
          // the leader's full barrier.
          const uint32_t fl = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * (Cfg::kAbTx + Cfg::kSfTx));
          tma_load_3d_pair(ssfa, &p.tm_sfa, fl, 0, mt * 2 + static_cast<int>(rank),
                           kb * Cfg::kSfChunks, pol);
          tma_load_3d_pair(ssfb, &p.tm_sfb, fl, 0, nt * 2, kb * Cfg::kSfChunks, pol);
          tma_load_2d_pair(sa, &p.tm_a, fl, kb * Cfg::kBKBytes,
                           mt * 2 * Cfg::kBM + static_cast<int>(rank) * Cfg::kBM, pol);
          tma_load_2d_pair(sb, &p.tm_b, fl, kb * Cfg::kBKBytes,
                           nt * Cfg::kBN + static_cast<int>(rank) * Cfg::kBNHalf, pol);
          continue;
        }
        const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[stage]), 0);
        if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::kAbTx);
        mbar_arrive_expect_tx(&sf_full[stage], Cfg::kSfTx);
        // Scales first: they are small, land early, and the stagers move them
        // into TMEM while A and B are still arriving.
        tma_load_3d(ssfa, &p.tm_sfa, &sf_full[stage], 0, mt * 2 + static_cast<int>(rank),
                    kb * Cfg::kSfChunks, pol);
        tma_load_3d(ssfb, &p.tm_sfb, &sf_full[stage], 0, nt * 2, kb * Cfg::kSfChunks, pol);
        tma_load_2d_pair(sa, &p.tm_a, full_leader, kb * Cfg::kBKBytes,
                         mt * 2 * Cfg::kBM + static_cast<int>(rank) * Cfg::kBM, pol);
        tma_load_2d_pair(sb, &p.tm_b, full_leader, kb * Cfg::kBKBytes,
                         nt * Cfg::kBN + static_cast<int>(rank) * Cfg::kBNHalf, pol);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      }
      if (!ok) {
        // Drain: every issued stage's copies land before the CTA retires its
        // shared memory.  Scale bytes land on this CTA's barriers; A/B bytes
        // on the leader's (the peer cannot observe those, so it waits).
        uint32_t dummy = 0;
        for (int s = 0; s < Cfg::kStages; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          mbar_wait_bounded(&sf_full[s], (issued_parity >> s) & 1u, p.timeout_ns, &dummy,
                            nullptr, 0);
          if (leader)
            mbar_wait_bounded(&full_bar[s], (issued_parity >> s) & 1u, p.timeout_ns, &dummy,
                              nullptr, 0);
        }
        if (!leader) spin_ns(200000);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (leader && lane == 0) {
      const uint32_t idesc_base =
          kFp4 ? make_idesc_block_scaled(2 * Cfg::kBM, Cfg::kBN, 1u, 0u, 0u, 0u)
               : make_idesc_block_scaled(2 * Cfg::kBM, Cfg::kBN, 0u, 1u, 0u, 0u);
      bool ok = true;
      int g = 0;
      for (int it = 0; it < my_tiles && ok; ++it) {
        if (!mbar_wait_bounded(acc_empty, (it & 1) ^ 1u, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int stage = g % Cfg::kStages;
          const uint32_t phase = static_cast<uint32_t>((g / Cfg::kStages) & 1);
          const bool cp_mode = (p.diag & 16u) != 0;
          if (!mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutMma) ||
              (!cp_mode && !mbar_wait_bounded(&sf_ready[stage], phase, p.timeout_ns, abort_flag,
                                              p.status, kDevTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          const uint32_t sfa_col = tmem_base + Cfg::kTmemSfBase + stage * Cfg::kTmemSfStageCols;
          const uint32_t sfb_col = sfa_col + Cfg::kSfaCols;
          if (cp_mode && !(p.diag & 1u)) {
            uint8_t* ssfa = sb + Cfg::kBBytes;
            uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
#pragma unroll
            for (int c = 0; c < Cfg::kSfChunks; ++c) {
              tmem_cp_pair_32x128b_warpx4(
                  sfa_col + c * 4, make_smem_desc(smem_u32(ssfa + c * 512), 0, 128, kSwizzleNone));
#pragma unroll
              for (int h = 0; h < 2; ++h)
                tmem_cp_pair_32x128b_warpx4(
                    sfb_col + c * 8 + h * 4,
                    make_smem_desc(smem_u32(ssfb + (c * 2 + h) * 512), 0, 128, kSwizzleNone));
            }
          }
          const uint64_t adesc = make_smem_desc(smem_u32(sa), 16, 1024, kSwizzle128B);
          const uint64_t bdesc = make_smem_desc(smem_u32(sb), 16, 1024, kSwizzle128B);
          if (!(p.diag & 2u)) {
#pragma unroll
            for (int j = 0; j < Cfg::kMmaPerStage; ++j) {
              const uint64_t koff = static_cast<uint64_t>(j * 2);  // +32 B of K
              const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
              if (kFp4) {
                mma_pair_mxf4nvf4(tmem_base, adesc + koff, bdesc + koff, idesc_base,
                                  sfa_col + j * 4, sfb_col + j * 8, acc);
              } else {
                const uint32_t idesc = idesc_base | (static_cast<uint32_t>(j) << 29) |
                                       (static_cast<uint32_t>(j) << 4);
                mma_pair_mxf8f6f4(tmem_base, adesc + koff, bdesc + koff, idesc, sfa_col,
                                  sfb_col, acc);
              }
            }
          }
          tc_commit_pair(&empty_bar[stage], 0x3);
        }
        if (ok) tc_commit_pair(acc_full, 0x3);
      }
      tc_commit_pair(drain_bar, 0x1);
      uint32_t dummy = 0;
      mbar_wait_bounded(drain_bar, 0, p.timeout_ns, &dummy, nullptr, 0);
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- scale stagers
    const int quad = warp % 4;
    const int stager_kb = (p.diag & 16u) ? 0 : total_kb;  // diag 64: stage, loads as cp mode
    const uint32_t t_quad = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    for (int g = 0; g < stager_kb; ++g) {
      const int stage = g % Cfg::kStages;
      const uint32_t phase = static_cast<uint32_t>((g / Cfg::kStages) & 1);
      // One lane polls the barrier; the warp follows it.
      bool ok = true;
      if (lane == 0 && !(p.diag & 32u))
        ok = mbar_wait_bounded(&sf_full[stage], phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      if (!(p.diag & 32u)) mbar_try_wait(&sf_full[stage], phase);  // acquire for every lane
      const uint8_t* ssfa = smem + stage * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes;
      const uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
      const uint32_t sfa_col = Cfg::kTmemSfBase + stage * Cfg::kTmemSfStageCols;
      if (!(p.diag & 1u)) {
        stage_scales<kFp4>(ssfa, ssfb, t_quad, sfa_col, sfa_col + Cfg::kSfaCols, lane);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      // A release-scoped arrive at cluster scope costs ~1 us here and serialises
      // the stagers (measured: 2.2 vs 4.1 PF/s).  The relaxed arrive is
      // enough: tcgen05.wait::st has already completed the TMEM writes and
      // tcgen05.fence::before_thread_sync orders them before the arrive.
      if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&sf_ready[stage]), 0));
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp % 4;
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(acc_empty), 0);
    float alpha = 1.0f;
    if (p.a_ts) alpha *= *p.a_ts;
    if (p.b_ts) alpha *= *p.b_ts;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    for (int it = 0; it < my_tiles; ++it) {
      const int tile = pair + it * npairs;
      const int mt = tile % p.num_m_tiles;
      const int nt = tile / p.num_m_tiles;
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded<false, 256>(acc_full, it & 1, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutEpilogue);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(acc_full, it & 1);
      tc_fence_after();
      const int row = mt * 2 * Cfg::kBM + static_cast<int>(rank) * Cfg::kBM + quad * 32 + lane;
      const bool row_ok = row < p.m && !(p.diag & 8u);
      const int n0 = nt * Cfg::kBN;
      if (kOutBf16 && p.vec_ok && n0 + Cfg::kBN <= p.n) {
        // Full tile: the whole accumulator row goes to registers as bf16,
        // the accumulator is handed back, then 16-byte stores.
        uint32_t packed[Cfg::kBN / 2];
#pragma unroll
        for (int cc = 0; cc < Cfg::kBN / 16; ++cc) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_row + cc * 16, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            packed[cc * 8 + j] = bf16x2_bits(__uint_as_float(r[2 * j]) * alpha,
                                             __uint_as_float(r[2 * j + 1]) * alpha);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.c) +
                                                row * p.ldc + n0);
#pragma unroll
          for (int v = 0; v < Cfg::kBN / 8; ++v)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2],
                                packed[4 * v + 3]);
        }
      } else {
        // fp32 output or a ragged tile: 32 columns at a time, accumulator
        // handed back after the last TMEM read.
#pragma unroll 1
        for (int cc = 0; cc < Cfg::kBN / 32; ++cc) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_row + cc * 32, r);
          tmem_wait_ld();
          if (cc == Cfg::kBN / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
          }
          const int col0 = n0 + cc * 32;
          if (row_ok && col0 < p.n) {
            const bool vec = p.vec_ok && col0 + 32 <= p.n;
            if (kOutBf16) {
              __nv_bfloat16* crow = reinterpret_cast<__nv_bfloat16*>(p.c) + row * p.ldc;
              if (vec) {
                uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
                for (int v = 0; v < 4; ++v)
                  dst[v] = make_uint4(bf16x2_bits(__uint_as_float(r[8 * v]) * alpha,
                                                  __uint_as_float(r[8 * v + 1]) * alpha),
                                      bf16x2_bits(__uint_as_float(r[8 * v + 2]) * alpha,
                                                  __uint_as_float(r[8 * v + 3]) * alpha),
                                      bf16x2_bits(__uint_as_float(r[8 * v + 4]) * alpha,
                                                  __uint_as_float(r[8 * v + 5]) * alpha),
                                      bf16x2_bits(__uint_as_float(r[8 * v + 6]) * alpha,
                                                  __uint_as_float(r[8 * v + 7]) * alpha));
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < p.n)
                    crow[col0 + j] = __float2bfloat16_rn(__uint_as_float(r[j]) * alpha);
              }
            } else {
              float* crow = reinterpret_cast<float*>(p.c) + row * p.ldc;
              if (vec) {
                float4* dst = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
                for (int v = 0; v < 8; ++v)
                  dst[v] = make_float4(__uint_as_float(r[v * 4]) * alpha,
                                       __uint_as_float(r[v * 4 + 1]) * alpha,
                                       __uint_as_float(r[v * 4 + 2]) * alpha,
                                       __uint_as_float(r[v * 4 + 3]) * alpha);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < p.n) crow[col0 + j] = __uint_as_float(r[j]) * alpha;
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // the leader's MMAs into both TMEMs are drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

template <bool kFp4, bool kOutBf16>
static cudaError_t launch_pair_one(const GemmParams& p, int grid, cudaStream_t stream) {
  using Cfg = PairCfg<kFp4>;
  auto kern = gemm_pair_kernel<kFp4, kOutBf16>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm_pair(const GemmParams& p, bool fp4, bool out_bf16, int grid,
                             cudaStream_t stream) {
  if (fp4) {
    return out_bf16 ? launch_pair_one<true, true>(p, grid, stream)
                    : launch_pair_one<true, false>(p, grid, stream);
  }
  return out_bf16 ? launch_pair_one<false, true>(p, grid, stream)
                  : launch_pair_one<false, false>(p, grid, stream);
}

int pair_tile_m() { return 2 * PairCfg<true>::kBM; }
int pair_tile_n() { return PairCfg<true>::kBN; }

}  // namespace qg
