// gemm_skinny.cu -- decode-shaped NVFP4 GEMM (few activation rows, large
// weight matrix), HBM-bound.
//
// C[m, n] = (ts_x * ts_w) * sum_k x(m,k) w(n,k), m <= 128, computed as
// C^T = W . X^T so the weight rows fill the tensor core's M = 128 side and the
// activation rows its N side (16 / 32 / 64 / 128).  The reference has no
// kernel for this shape (its harness only runs square problems,
// GEMMquant_sm110/src/quant_gemm_bench.cu:3038-3079); BASELINE config 4 names
// it.  The weights are streamed once from HBM; every CTA takes an equal,
// contiguous range of (weight-tile, K-block) units ("stream-K"), so the
// 224 x 32 units of N = 28672, K = 8192 spread evenly over 148 SMs.  A tile
// that one CTA owns is scaled and written to C by that CTA; a tile split
// between CTAs is summed by the last of them to finish (see the epilogue).
// The grid is a programmatic dependent of the activation quantizer
// (skinny_quant.cu), so no memset, reduction or finishing launch is needed.
//
// Roles (10 warps): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2..5 epilogue (one TMEM quadrant each: lane = weight row), warps 6..9
// scale stagers (tcgen05.st, as in gemm_solo.cu).  The accumulator is double
// buffered so a segment's reduction overlaps the next segment's mainloop.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

// Upper bound of the GEMM grid; sizes the partial-tile workspace.
constexpr int kSkinnyMaxCtas = 256;

template <int kN>
struct SkinnyCfg {
  static constexpr int kBM = 128;       // weight rows per tile
  static constexpr int kBKBytes = 128;  // 256 fp4 of K per stage
  static constexpr int kStages = kN >= 128 ? 6 : 8;
  static constexpr int kMmaPerStage = 4;
  static constexpr int kSfChunks = 4;
  static constexpr int kWBytes = kBM * kBKBytes;
  static constexpr int kXBytes = kN * kBKBytes;
  static constexpr int kSfwBytes = kSfChunks * 512;
  static constexpr int kSfxBytes = kSfChunks * 512;
  static constexpr int kStageTx = kWBytes + kXBytes + kSfwBytes + kSfxBytes;
  static constexpr int kStageBytes = (kStageTx + 1023) / 1024 * 1024;
  static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
  static constexpr int kSfStageCols = 32;  // 16 weight + 16 activation
  static constexpr int kTmemSfBase = 256;
  static constexpr int kTmemCols = 512;
  static_assert(2 * kN <= kTmemSfBase, "accumulators");
  static_assert(kTmemSfBase + kStages * kSfStageCols <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr int kThreads = 320;
};

// Walk of one CTA's unit range: a "segment" is a run of K-blocks of one tile.
struct UnitRange {
  int u0, u1, nkb;
};

// Diagnostic stamp (QG_DIAG_FLAGS bit 6): CTA 0 writes %globaltimer into
// slot `i` of the last (never used by a launched CTA) partial slice pair.
__device__ __forceinline__ void trace(const SkinnyParams& p, int i) {
  if ((p.diag & 64u) && blockIdx.x == 0 && i < 512)
    reinterpret_cast<unsigned long long*>(p.part + static_cast<int64_t>(kSkinnyMaxCtas - 1) * 2 * p.m * 128)[i] = globaltimer_ns();
}

template <int kN>
__global__ void __launch_bounds__(320, 1) gemm_skinny_kernel(const __grid_constant__ SkinnyParams p) {
  using Cfg = SkinnyCfg<kN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* sf_ready = bars + Cfg::kStages;
  uint64_t* empty_bar = bars + 2 * Cfg::kStages;
  uint64_t* acc_full = bars + 3 * Cfg::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;            // [2]
  uint64_t* drain_bar = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 5);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&sf_ready[s], 4);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    fence_barrier_init();
    tma_prefetch_desc(&p.tm_w);
    tma_prefetch_desc(&p.tm_x);
    tma_prefetch_desc(&p.tm_sfw);
    tma_prefetch_desc(&p.tm_sfx);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (threadIdx.x == 0) trace(p, 0);
  const int64_t units = static_cast<int64_t>(p.num_tiles) * p.num_k_blocks;
  UnitRange ur;
  ur.u0 = static_cast<int>(units * blockIdx.x / gridDim.x);
  ur.u1 = static_cast<int>(units * (blockIdx.x + 1) / gridDim.x);
  ur.nkb = p.num_k_blocks;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();  // weights: streamed once
      const uint64_t pol_x = l2_policy_evict_last();   // activations: reused by all CTAs
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      int stage = 0, tile = ur.u0 / ur.nkb, kb = ur.u0 % ur.nkb;
      uint32_t phase = 0;
      // The first kStages stages get their weight loads at once; their
      // activation loads wait for the quantizer grid (griddep_wait), so the
      // weight stream starts while the activations are being quantised.
      int deferred = 0;
      int dkb[Cfg::kStages];
      auto issue_x = [&](int s, int k_blk) {
        uint8_t* sx = smem + s * Cfg::kStageBytes + Cfg::kWBytes;
        uint8_t* ssfx = sx + Cfg::kXBytes + Cfg::kSfwBytes;
        tma_load_3d(ssfx, &p.tm_sfx, &full_bar[s], 0, 0, k_blk * Cfg::kSfChunks, pol_x);
        tma_load_2d(sx, &p.tm_x, &full_bar[s], k_blk * Cfg::kBKBytes, 0, pol_x);
      };
      bool dep_done = false;
      auto release_deferred = [&]() {
        griddep_wait();
        trace(p, 2);
        for (int s = 0; s < deferred; ++s) issue_x(s, dkb[s]);
        dep_done = true;
      };
      for (int u = ur.u0, g = 0; u < ur.u1; ++u, ++g) {
        if (!dep_done && g == Cfg::kStages) release_deferred();
        if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* sw = smem + stage * Cfg::kStageBytes;
        uint8_t* ssfw = sw + Cfg::kWBytes + Cfg::kXBytes;
        trace(p, 16 + g);
        mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageTx);
        tma_load_3d(ssfw, &p.tm_sfw, &full_bar[stage], 0, tile, kb * Cfg::kSfChunks, pol_w);
        tma_load_2d(sw, &p.tm_w, &full_bar[stage], kb * Cfg::kBKBytes, tile * Cfg::kBM, pol_w);
        if (dep_done) {
          issue_x(stage, kb);
        } else {
          dkb[deferred++] = kb;
        }
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++kb == ur.nkb) {
          kb = 0;
          ++tile;
        }
        if (++stage == Cfg::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!dep_done) release_deferred();
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
      // The issue loop is the kernel's serial path: counters are stepped
      // incrementally and descriptors offset by constants, so no division or
      // modulo runs per unit.
      const uint32_t idesc = make_idesc_block_scaled(Cfg::kBM, kN, 1u, 0u, 0u, 0u);
      const uint64_t wdesc0 = make_smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      const uint64_t xdesc0 = make_smem_desc(smem_u32(smem + Cfg::kWBytes), 16, 1024, kSwizzle128B);
      constexpr uint64_t kStageDesc = Cfg::kStageBytes >> 4;
      bool ok = true;
      int seg = 0, stage = 0, kb = ur.u0 % ur.nkb;
      uint32_t phase = 0, acc = 0;
      for (int u = ur.u0; u < ur.u1 && ok; ++u) {
        const int buf = seg & 1;
        if (u == ur.u0 || kb == 0) {
          if (!mbar_wait_bounded(&acc_empty[buf], ((seg >> 1) & 1) ^ 1u, p.timeout_ns, abort_flag,
                                 p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          acc = 0;
        }
        if (!mbar_wait_bounded(&sf_ready[stage], phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma) ||
            !mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sfw_col = tmem_base + Cfg::kTmemSfBase + stage * Cfg::kSfStageCols;
        const uint64_t wdesc = wdesc0 + stage * kStageDesc;
        const uint64_t xdesc = xdesc0 + stage * kStageDesc;
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kN);
#pragma unroll
        for (int j = 0; j < Cfg::kMmaPerStage; ++j) {
          const uint64_t koff = static_cast<uint64_t>(j * 2);
          mma_mxf4nvf4(d_tmem, wdesc + koff, xdesc + koff, idesc, sfw_col + j * 4,
                       sfw_col + 16 + j * 4, acc);
          acc = 1;
        }
        tc_commit(&empty_bar[stage]);
        if (u == ur.u1 - 1 || kb == ur.nkb - 1) {
          tc_commit(&acc_full[buf]);
          ++seg;
        }
        if (++kb == ur.nkb) kb = 0;
        if (++stage == Cfg::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      tc_commit(drain_bar);
      uint32_t dummy = 0;
      mbar_wait_bounded(drain_bar, 0, p.timeout_ns, &dummy, nullptr, 0);
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- scale stagers
    const int quad = warp % 4;
    const uint32_t t_quad = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    int stage = 0;
    uint32_t phase = 0;
    for (int u = ur.u0; u < ur.u1; ++u) {
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(&full_bar[stage], phase);
      const uint8_t* ssfw = smem + stage * Cfg::kStageBytes + Cfg::kWBytes + Cfg::kXBytes;
      const uint8_t* ssfx = ssfw + Cfg::kSfwBytes;
      uint32_t a[16], b[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = lds128(ssfw + c * 512 + lane * 16);
        const uint4 w = lds128(ssfx + c * 512 + lane * 16);
        a[4 * c] = v.x; a[4 * c + 1] = v.y; a[4 * c + 2] = v.z; a[4 * c + 3] = v.w;
        b[4 * c] = w.x; b[4 * c + 1] = w.y; b[4 * c + 2] = w.z; b[4 * c + 3] = w.w;
      }
      const uint32_t col = Cfg::kTmemSfBase + stage * Cfg::kSfStageCols;
      tmem_st_32x32b<16>(t_quad + col, a);
      tmem_st_32x32b<16>(t_quad + col + 16, b);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sf_ready[stage]);
      if (++stage == Cfg::kStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // Lane = weight row = output column n; the kN accumulator columns are the
    // activation rows m.  A tile owned by one CTA is scaled and stored to C.
    // A split tile: every contributor stores its partial to its own slice,
    // then bumps the tile's counter (one per TMEM quadrant); the last to
    // arrive sums the slices in contributor order, so the result does not
    // depend on which CTA finished last.
    const int quad = warp % 4;
    const uint32_t t_quad = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    griddep_wait();  // the tensor scale and the counters come from the quantizer grid
    if (quad == 0 && lane == 0) trace(p, 3);
    const float alpha = (p.x_ts ? *p.x_ts : 1.0f) * (p.w_ts ? *p.w_ts : 1.0f);
    const int64_t units_all = static_cast<int64_t>(p.num_tiles) * ur.nkb;
    const int64_t grid = gridDim.x;
    auto contributor = [&](int64_t u) { return static_cast<int>(((u + 1) * grid - 1) / units_all); };
    auto first_tile = [&](int c) { return static_cast<int>(units_all * c / grid / ur.nkb); };
    auto store_c = [&](int m, int n, float v) {
      if (p.out_bf16)
        reinterpret_cast<__nv_bfloat16*>(p.c)[static_cast<int64_t>(m) * p.ldc + n] =
            __float2bfloat16_rn(v);
      else
        reinterpret_cast<float*>(p.c)[static_cast<int64_t>(m) * p.ldc + n] = v;
    };
    const int tile_lo = ur.u0 / ur.nkb, tile_hi = (ur.u1 - 1) / ur.nkb;
    const int my_first = tile_lo;
    for (int t = tile_lo, seg = 0; t <= tile_hi; ++t, ++seg) {
      const int buf = seg & 1;
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded<false, 128>(&acc_full[buf], (seg >> 1) & 1, p.timeout_ns,
                                           abort_flag, p.status, kDevTimeoutEpilogue);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(&acc_full[buf], (seg >> 1) & 1);
      tc_fence_after();
      const int col = quad * 32 + lane;
      const int n = t * Cfg::kBM + col;
      const bool n_ok = n < p.n;
      const int cf = contributor(static_cast<int64_t>(t) * ur.nkb);
      const int cl = contributor(static_cast<int64_t>(t + 1) * ur.nkb - 1);
      float* mine = p.part + static_cast<int64_t>(blockIdx.x * 2 + (t == my_first ? 0 : 1)) *
                                 p.m * Cfg::kBM;
#pragma unroll
      for (int cc = 0; cc < kN / 16; ++cc) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_quad + static_cast<uint32_t>(buf * kN + cc * 16), r);
        tmem_wait_ld();
        if (cc == kN / 16 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = cc * 16 + j;
          if (m < p.m) {
            const float v = __uint_as_float(r[j]);
            if (cf == cl) {
              if (n_ok) store_c(m, n, v * alpha);
            } else {
              __stcg(mine + m * Cfg::kBM + col, v);
            }
          }
        }
      }
      if (quad == 0 && lane == 0) trace(p, 100 + seg);
      if (cf == cl) continue;
      __threadfence();
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atomicAdd(&p.cnt[t * 4 + quad], 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old != static_cast<uint32_t>(cl - cf)) continue;
      __threadfence();
      // Sum pass: a lane takes 4 adjacent columns of one row, a warp
      // instruction 4 rows x 32 columns; 8 instructions x 2 contributors of
      // 16-byte loads are in flight per warp before the adds, in order.
      {
        const int sub = lane >> 3, c4 = (lane & 7) * 4;
        const int64_t slice = static_cast<int64_t>(p.m) * Cfg::kBM;
        for (int m0 = 0; m0 < p.m; m0 += 32) {
          float4 acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int c = cf; c <= cl; c += 2) {
            const bool two = c + 1 <= cl;
            const float* s0 = p.part + (c * 2 + (t == first_tile(c) ? 0 : 1)) * slice + quad * 32 + c4;
            const float* s1 = two ? p.part + ((c + 1) * 2 + (t == first_tile(c + 1) ? 0 : 1)) * slice +
                                        quad * 32 + c4
                                  : s0;
            float4 v0[8], v1[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int m = m0 + i * 4 + sub;
              const bool ok = m < p.m;
              v0[i] = ok ? __ldcg(reinterpret_cast<const float4*>(s0 + m * Cfg::kBM))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
              v1[i] = ok && two ? __ldcg(reinterpret_cast<const float4*>(s1 + m * Cfg::kBM))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              acc[i].x += v0[i].x; acc[i].y += v0[i].y; acc[i].z += v0[i].z; acc[i].w += v0[i].w;
              if (two) {
                acc[i].x += v1[i].x; acc[i].y += v1[i].y; acc[i].z += v1[i].z; acc[i].w += v1[i].w;
              }
            }
          }
          const int nb = t * Cfg::kBM + quad * 32 + c4;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int m = m0 + i * 4 + sub;
            if (m >= p.m) continue;
            const float e[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (nb + q < p.n) store_c(m, nb + q, e[q] * alpha);
          }
        }
      }
      if (lane == 0) p.cnt[t * 4 + quad] = 0u;  // ready for the next call
      if (quad == 0 && lane == 0) trace(p, 200 + seg);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace(p, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

template <int kN>
static cudaError_t launch_skinny_n(const SkinnyParams& p, int grid, cudaStream_t stream) {
  using Cfg = SkinnyCfg<kN>;
  auto kern = gemm_skinny_kernel<kN>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

int skinny_max_ctas() { return kSkinnyMaxCtas; }

int skinny_mma_n(int64_t m) { return m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128; }

cudaError_t launch_gemm_skinny(const SkinnyParams& p, int grid, cudaStream_t stream) {
  switch (skinny_mma_n(p.m)) {
    case 16: return launch_skinny_n<16>(p, grid, stream);
    case 32: return launch_skinny_n<32>(p, grid, stream);
    case 64: return launch_skinny_n<64>(p, grid, stream);
    default: return launch_skinny_n<128>(p, grid, stream);
  }
}

}  // namespace qg
