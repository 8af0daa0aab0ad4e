// gemm_blockscaled.cu -- persistent tcgen05 block-scaled GEMM for sm_100a.
//
// C[M,N] = alpha * A[M,K] . B[N,K]^T with per-block scale factors, for
//   NVFP4: kind::mxf4nvf4.block16 (e2m1 values, ue4m3 scale per 16 K)
//   MXFP8: kind::mxf8f6f4          (e4m3 values, ue8m0 scale per 32 K)
// This is the B200 replacement for the reference's NVFP4 GEMM backends
// (CUTLASS example 72b, GEMMquant_sm110/build_and_run.sh:38-75, and the tc6
// runner, GEMMsm110/include/backends/tc6_nvfp4.cuh:334-559, whose mainloop was
// FP16).
//
// One CTA per SM, persistent over 128 x 256 output tiles:
//   warp 0      TMA producer: A, B (SWIZZLE_128B) and their scale chunks into
//               a kStages-deep shared-memory ring guarded by mbarriers.
//   warp 1      TMEM owner + MMA issuer: copies each stage's scale chunks to
//               TMEM (tcgen05.cp 32x128b.warpx4), issues 4 MMAs (K = 64 fp4 /
//               32 fp8 each), commits the stage back to the producer.
//   warps 2..5  epilogue: tcgen05.ld the fp32 accumulator (one 32-lane TMEM
//               quadrant per warp), hand the accumulator back, scale by alpha,
//               convert and store.
// Every wait is bounded (qg_ptx.cuh); on expiry the CTA drains its in-flight
// copies and MMAs, frees TMEM and exits with a status code.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

template <bool kFp4>
struct TileCfg {
  static constexpr int kBM = 128;
  static constexpr int kBN = 256;
  static constexpr int kBKBytes = 128;  // one SWIZZLE_128B row per stage
  static constexpr int kStages = 4;
  static constexpr int kMmaPerStage = 4;  // 32 bytes of K per MMA
  // Scale chunks (512 B = 128 rows x 4 scales) along K per stage.
  static constexpr int kSfChunks = kFp4 ? 4 : 1;
  static constexpr int kABytes = kBM * kBKBytes;
  static constexpr int kBBytes = kBN * kBKBytes;
  static constexpr int kSfaBytes = kSfChunks * 512 * (kBM / 128);
  static constexpr int kSfbBytes = kSfChunks * 512 * (kBN / 128);
  static constexpr int kStageTx = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  // Stage bases stay 1024-byte aligned (SWIZZLE_128B atom).
  static constexpr int kStageBytes = (kStageTx + 1023) / 1024 * 1024;
  static constexpr int kSmemBytes = kStages * kStageBytes + 256 /*barriers*/ + 1024 /*align*/;
  // TMEM columns: accumulator [0, kBN), then per-stage scale slots.
  static constexpr int kSfaCols = kSfChunks * 4;
  static constexpr int kSfbCols = kSfChunks * 4 * (kBN / 128);
  static constexpr int kTmemSfBase = kBN;
  static constexpr int kTmemSfStageCols = kSfaCols + kSfbCols;
  static constexpr int kTmemCols = 512;
  static_assert(kTmemSfBase + kStages * kTmemSfStageCols <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr int kThreads = 192;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Store 32 consecutive accumulator columns of one output row.
template <bool kOutBf16>
__device__ __forceinline__ void store_run(const GemmParams& p, int row, int col0,
                                          const uint32_t (&r)[32], float alpha) {
  if (kOutBf16) {
    __nv_bfloat16* crow = reinterpret_cast<__nv_bfloat16*>(p.c) + row * p.ldc;
    if (p.vec_ok && col0 + 32 <= p.n) {
      uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[v * 8 + 0]) * alpha, __uint_as_float(r[v * 8 + 1]) * alpha);
        w.y = pack_bf16x2(__uint_as_float(r[v * 8 + 2]) * alpha, __uint_as_float(r[v * 8 + 3]) * alpha);
        w.z = pack_bf16x2(__uint_as_float(r[v * 8 + 4]) * alpha, __uint_as_float(r[v * 8 + 5]) * alpha);
        w.w = pack_bf16x2(__uint_as_float(r[v * 8 + 6]) * alpha, __uint_as_float(r[v * 8 + 7]) * alpha);
        dst[v] = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.n) crow[col0 + j] = __float2bfloat16_rn(__uint_as_float(r[j]) * alpha);
    }
  } else {
    float* crow = reinterpret_cast<float*>(p.c) + row * p.ldc;
    if (p.vec_ok && col0 + 32 <= p.n) {
      float4* dst = reinterpret_cast<float4*>(crow + col0);
#pragma unroll
      for (int v = 0; v < 8; ++v)
        dst[v] = make_float4(__uint_as_float(r[v * 4 + 0]) * alpha, __uint_as_float(r[v * 4 + 1]) * alpha,
                             __uint_as_float(r[v * 4 + 2]) * alpha, __uint_as_float(r[v * 4 + 3]) * alpha);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.n) crow[col0 + j] = __uint_as_float(r[j]) * alpha;
    }
  }
}

template <bool kFp4, bool kOutBf16>
__global__ void __launch_bounds__(192, 1)
    gemm_blockscaled_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = TileCfg<kFp4>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + Cfg::kStages;
  uint64_t* acc_full = bars + 2 * Cfg::kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain_bar = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 3);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
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

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mt = tile % p.num_m_tiles;
        const int nt = tile / p.num_m_tiles;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          uint8_t* ssfa = sb + Cfg::kBBytes;
          uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageTx);
          tma_load_2d(sa, &p.tm_a, &full_bar[stage], kb * Cfg::kBKBytes, mt * Cfg::kBM, pol_a);
          tma_load_2d(sb, &p.tm_b, &full_bar[stage], kb * Cfg::kBKBytes, nt * Cfg::kBN, pol_a);
          tma_load_3d(ssfa, &p.tm_sfa, &full_bar[stage], 0, mt * (Cfg::kBM / 128),
                      kb * Cfg::kSfChunks, pol_a);
          tma_load_3d(ssfb, &p.tm_sfb, &full_bar[stage], 0, nt * (Cfg::kBN / 128),
                      kb * Cfg::kSfChunks, pol_a);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: every issued stage's bytes must land before the CTA exits.
        for (int s = 0; s < Cfg::kStages; ++s) {
          if (issued_mask & (1u << s)) {
            uint32_t dummy = 0;
            mbar_wait_bounded(&full_bar[s], (issued_parity >> s) & 1u, p.timeout_ns, &dummy,
                              nullptr, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      const uint32_t idesc_base =
          kFp4 ? make_idesc_block_scaled(Cfg::kBM, Cfg::kBN, 1u, 0u, 0u, 0u)
               : make_idesc_block_scaled(Cfg::kBM, Cfg::kBN, 0u, 1u, 0u, 0u);
      const uint32_t acc_tmem = tmem_base;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        if (!mbar_wait_bounded(acc_empty, (it & 1) ^ 1u, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          uint8_t* ssfa = sb + Cfg::kBBytes;
          uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
          const uint32_t sf_col = tmem_base + Cfg::kTmemSfBase + stage * Cfg::kTmemSfStageCols;
          const uint32_t sfa_col = sf_col;
          const uint32_t sfb_col = sf_col + Cfg::kSfaCols;
          // Scale chunks -> TMEM.  A chunk c covers 128 rows x 4 scales; it
          // lands in 4 columns (row r at lane r%32 of every quadrant, column
          // r/32, byte = scale index).
          for (int c = 0; c < Cfg::kSfChunks; ++c) {
            tmem_cp_32x128b_warpx4(sfa_col + c * 4,
                                   make_smem_desc(smem_u32(ssfa + c * 512), 0, 128, kSwizzleNone));
#pragma unroll
            for (int b = 0; b < Cfg::kBN / 128; ++b) {
              tmem_cp_32x128b_warpx4(
                  sfb_col + c * 4 * (Cfg::kBN / 128) + b * 4,
                  make_smem_desc(smem_u32(ssfb + (c * (Cfg::kBN / 128) + b) * 512), 0, 128,
                                 kSwizzleNone));
            }
          }
          const uint64_t adesc = make_smem_desc(smem_u32(sa), 16, 1024, kSwizzle128B);
          const uint64_t bdesc = make_smem_desc(smem_u32(sb), 16, 1024, kSwizzle128B);
#pragma unroll
          for (int j = 0; j < Cfg::kMmaPerStage; ++j) {
            // +32 bytes of K inside the 128-byte swizzle row (>> 4 -> +2).
            const uint64_t koff = static_cast<uint64_t>(j * 2);
            const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
            if (kFp4) {
              mma_mxf4nvf4(acc_tmem, adesc + koff, bdesc + koff, idesc_base,
                           sfa_col + j * 4, sfb_col + j * 4 * (Cfg::kBN / 128), acc);
            } else {
              const uint32_t idesc = idesc_base | (static_cast<uint32_t>(j) << 29) |
                                     (static_cast<uint32_t>(j) << 4);
              mma_mxf8f6f4(acc_tmem, adesc + koff, bdesc + koff, idesc, sfa_col, sfb_col, acc);
            }
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) tc_commit(acc_full);
      }
      // Drain: all issued tcgen05 work completes before TMEM is released.
      tc_commit(drain_bar);
      uint32_t dummy = 0;
      mbar_wait_bounded(drain_bar, 0, p.timeout_ns, &dummy, nullptr, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp % 4;  // TMEM lanes [32*quad, 32*quad + 32)
    float alpha = 1.0f;
    if (p.a_ts) alpha *= *p.a_ts;
    if (p.b_ts) alpha *= *p.b_ts;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int mt = tile % p.num_m_tiles;
      const int nt = tile / p.num_m_tiles;
      if (!mbar_wait_bounded(acc_full, it & 1, p.timeout_ns, abort_flag, p.status,
                             kDevTimeoutEpilogue))
        break;
      tc_fence_after();
      const int row = mt * Cfg::kBM + quad * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll 1
      for (int cc = 0; cc < Cfg::kBN / 32; ++cc) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld_32x32b_x32(t_row + cc * 32, r);
        tmem_wait_ld();
        if (cc == Cfg::kBN / 32 - 1) {
          // Whole accumulator read: hand it back to the MMA warp now so the
          // next tile's mainloop overlaps this tile's last stores.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty);
        }
        const int col0 = nt * Cfg::kBN + cc * 32;
        if (row < p.m && col0 < p.n) store_run<kOutBf16>(p, row, col0, r, alpha);
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
static cudaError_t launch_one(const GemmParams& p, int grid, cudaStream_t stream) {
  using Cfg = TileCfg<kFp4>;
  auto kern = gemm_blockscaled_kernel<kFp4, kOutBf16>;
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

cudaError_t launch_gemm_blockscaled(const GemmParams& p, bool fp4, bool out_bf16, int grid,
                                    cudaStream_t stream) {
  if (fp4) {
    return out_bf16 ? launch_one<true, true>(p, grid, stream)
                    : launch_one<true, false>(p, grid, stream);
  }
  return out_bf16 ? launch_one<false, true>(p, grid, stream)
                  : launch_one<false, false>(p, grid, stream);
}

int gemm_tile_m() { return TileCfg<true>::kBM; }
int gemm_tile_n() { return TileCfg<true>::kBN; }
int gemm_stage_k_bytes() { return TileCfg<true>::kBKBytes; }
int gemm_sf_chunks_per_stage(bool fp4) {
  return fp4 ? TileCfg<true>::kSfChunks : TileCfg<false>::kSfChunks;
}

}  // namespace qg
