// gemm_solo.cu -- persistent single-CTA block-scaled GEMM with TMEM scale
// staging by tcgen05.st.
//
// C[M,N] = alpha * A[M,K] . B[N,K]^T for NVFP4 (kind::mxf4nvf4.block16) and
// MXFP8 (kind::mxf8f6f4.block_scale): the B200 replacement for the
// reference's NVFP4 GEMM backends (CUTLASS example 72b,
// GEMMquant_sm110/build_and_run.sh:38-75; tc6,
// GEMMsm110/include/backends/tc6_nvfp4.cuh:334-559).
//
// One CTA per SM, persistent over 128 x 256 output tiles.  Scale factors
// reach TMEM through tcgen05.st by four stager warps (one per 32-lane TMEM
// quadrant) instead of tcgen05.cp: copies run in the tensor pipe in order
// with the MMAs at a roughly fixed cost each (12 per NVFP4 stage), which
// measured at ~40% of the kernel.  With one CTA the stagers hand off to the
// MMA issuer through a CTA-local barrier.
//
// Roles (10 warps):
//   warp 0      TMA producer (A, B SWIZZLE_128B; scale chunks via a 3-D map).
//   warp 1      TMEM owner + MMA issuer (4 MMAs per stage).
//   warps 2..5  epilogue: bf16 rows converted into registers, accumulator
//               handed back, then stored (fp32 / ragged: 32 columns at a time).
//   warps 6..9  scale stagers: shared memory -> registers -> TMEM, the layout
//               the MMA reads (row r at lane r%32 of every quadrant, column
//               r/32, byte = scale index).
// Every wait is bounded (qg_ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

template <bool kFp4>
struct SoloCfg {
  static constexpr int kBM = 128;
  static constexpr int kBN = 256;
  static constexpr int kBKBytes = 128;
  static constexpr int kStages = 4;
  static constexpr int kMmaPerStage = 4;
  static constexpr int kSfChunks = kFp4 ? 4 : 1;
  static constexpr int kABytes = kBM * kBKBytes;
  static constexpr int kBBytes = kBN * kBKBytes;
  static constexpr int kSfaBytes = kSfChunks * 512;
  static constexpr int kSfbBytes = kSfChunks * 512 * 2;
  static constexpr int kStageTx = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr int kStageBytes = (kStageTx + 1023) / 1024 * 1024;
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

__device__ __forceinline__ uint32_t bf16x2_bits_solo(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One stage's scales of this warp's TMEM quadrant: SFA chunks (4 columns
// each, the 16-byte row r of a chunk holds rows r, r+32, r+64, r+96) and the
// two 128-row SFB blocks per chunk (8 columns per chunk).
template <bool kFp4>
__device__ __forceinline__ void stage_scales_solo(const uint8_t* ssfa, const uint8_t* ssfb,
                                             uint32_t t_quad, uint32_t sfa_col, uint32_t sfb_col,
                                             int lane) {
  using Cfg = SoloCfg<kFp4>;
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
__global__ void __launch_bounds__(320, 1)
    gemm_solo_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = SoloCfg<kFp4>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* sf_ready = bars + Cfg::kStages;
  uint64_t* empty_bar = bars + 2 * Cfg::kStages;
  uint64_t* acc_full = bars + 3 * Cfg::kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain_bar = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 3);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&sf_ready[s], 4);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    fence_barrier_init();
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
    tma_prefetch_desc(&p.tm_sfa);
    tma_prefetch_desc(&p.tm_sfb);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  const int nkb = p.num_k_blocks;
  const int cta = static_cast<int>(blockIdx.x);
  const int ncta = static_cast<int>(gridDim.x);
  const int my_tiles = cta < num_tiles ? (num_tiles - 1 - cta) / ncta + 1 : 0;
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
        const int tile = cta + (g / nkb) * ncta;
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
        if (kDiag & 4u) {
          mbar_arrive(&full_bar[stage]);
          continue;
        }
        mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageTx);
        tma_load_3d(ssfa, &p.tm_sfa, &full_bar[stage], 0, mt, kb * Cfg::kSfChunks, pol);
        tma_load_3d(ssfb, &p.tm_sfb, &full_bar[stage], 0, nt * 2, kb * Cfg::kSfChunks, pol);
        tma_load_2d(sa, &p.tm_a, &full_bar[stage], kb * Cfg::kBKBytes, mt * Cfg::kBM, pol);
        tma_load_2d(sb, &p.tm_b, &full_bar[stage], kb * Cfg::kBKBytes, nt * Cfg::kBN, pol);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      }
      if (!ok) {
        uint32_t dummy = 0;
        for (int s = 0; s < Cfg::kStages; ++s)
          if (issued_mask & (1u << s))
            mbar_wait_bounded(&full_bar[s], (issued_parity >> s) & 1u, p.timeout_ns, &dummy,
                              nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc_base =
          kFp4 ? make_idesc_block_scaled(Cfg::kBM, Cfg::kBN, 1u, 0u, 0u, 0u)
               : make_idesc_block_scaled(Cfg::kBM, Cfg::kBN, 0u, 1u, 0u, 0u);
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
          if (!mbar_wait_bounded(&sf_ready[stage], phase, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutMma) ||
              !mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          const uint32_t sfa_col = tmem_base + Cfg::kTmemSfBase + stage * Cfg::kTmemSfStageCols;
          const uint32_t sfb_col = sfa_col + Cfg::kSfaCols;
          const uint64_t adesc = make_smem_desc(smem_u32(sa), 16, 1024, kSwizzle128B);
          const uint64_t bdesc = make_smem_desc(smem_u32(sb), 16, 1024, kSwizzle128B);
          if (!(kDiag & 2u)) {
#pragma unroll
            for (int j = 0; j < Cfg::kMmaPerStage; ++j) {
              const uint64_t koff = static_cast<uint64_t>(j * 2);  // +32 B of K
              const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
              if (kFp4) {
                mma_mxf4nvf4(tmem_base, adesc + koff, bdesc + koff, idesc_base, sfa_col + j * 4,
                             sfb_col + j * 8, acc);
              } else {
                const uint32_t idesc = idesc_base | (static_cast<uint32_t>(j) << 29) |
                                       (static_cast<uint32_t>(j) << 4);
                mma_mxf8f6f4(tmem_base, adesc + koff, bdesc + koff, idesc, sfa_col, sfb_col, acc);
              }
            }
          }
          tc_commit(&empty_bar[stage]);
        }
        if (ok) tc_commit(acc_full);
      }
      tc_commit(drain_bar);
      uint32_t dummy = 0;
      mbar_wait_bounded(drain_bar, 0, p.timeout_ns, &dummy, nullptr, 0);
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- scale stagers
    const int quad = warp % 4;
    const uint32_t t_quad = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    for (int g = 0; g < total_kb; ++g) {
      const int stage = g % Cfg::kStages;
      const uint32_t phase = static_cast<uint32_t>((g / Cfg::kStages) & 1);
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag,
                                          p.status, kDevTimeoutMma);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(&full_bar[stage], phase);  // acquire for every lane
      const uint8_t* ssfa = smem + stage * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes;
      const uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
      const uint32_t sfa_col = Cfg::kTmemSfBase + stage * Cfg::kTmemSfStageCols;
      if (!(kDiag & 1u)) {
        stage_scales_solo<kFp4>(ssfa, ssfb, t_quad, sfa_col, sfa_col + Cfg::kSfaCols, lane);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sf_ready[stage]);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp % 4;
    float alpha = 1.0f;
    if (p.a_ts) alpha *= *p.a_ts;
    if (p.b_ts) alpha *= *p.b_ts;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    for (int it = 0; it < my_tiles; ++it) {
      const int tile = static_cast<int>(blockIdx.x) + it * static_cast<int>(gridDim.x);
      const int mt = tile % p.num_m_tiles;
      const int nt = tile / p.num_m_tiles;
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded<false, 256>(acc_full, it & 1, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutEpilogue);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(acc_full, it & 1);
      tc_fence_after();
      const int row = mt * Cfg::kBM + quad * 32 + lane;
      const bool row_ok = row < p.m && !(kDiag & 8u);
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
            packed[cc * 8 + j] = bf16x2_bits_solo(__uint_as_float(r[2 * j]) * alpha,
                                             __uint_as_float(r[2 * j + 1]) * alpha);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);
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
            if (lane == 0) mbar_arrive(acc_empty);
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
                  dst[v] = make_uint4(bf16x2_bits_solo(__uint_as_float(r[8 * v]) * alpha,
                                                  __uint_as_float(r[8 * v + 1]) * alpha),
                                      bf16x2_bits_solo(__uint_as_float(r[8 * v + 2]) * alpha,
                                                  __uint_as_float(r[8 * v + 3]) * alpha),
                                      bf16x2_bits_solo(__uint_as_float(r[8 * v + 4]) * alpha,
                                                  __uint_as_float(r[8 * v + 5]) * alpha),
                                      bf16x2_bits_solo(__uint_as_float(r[8 * v + 6]) * alpha,
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
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

template <bool kFp4, bool kOutBf16>
static cudaError_t launch_solo_one(const GemmParams& p, int grid, cudaStream_t stream) {
  using Cfg = SoloCfg<kFp4>;
  auto kern = gemm_solo_kernel<kFp4, kOutBf16>;
  // The attribute belongs to the function in each device's context.
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm_solo(const GemmParams& p, bool fp4, bool out_bf16, int grid,
                             cudaStream_t stream) {
  if (fp4) {
    return out_bf16 ? launch_solo_one<true, true>(p, grid, stream)
                    : launch_solo_one<true, false>(p, grid, stream);
  }
  return out_bf16 ? launch_solo_one<false, true>(p, grid, stream)
                  : launch_solo_one<false, false>(p, grid, stream);
}

}  // namespace qg
