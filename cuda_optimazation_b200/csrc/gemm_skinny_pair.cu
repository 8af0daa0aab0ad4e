// gemm_skinny_pair.cu -- decode-shaped NVFP4 GEMM on CTA pairs (cta_group::2)
// for 33..128 activation rows, one whole 512-row weight tile per pair.
//
// C^T = W . X^T as in gemm_skinny.cu (weights on the MMA's M side, the
// activation rows on its N side), with the MMA issued for a CTA pair: one
// tcgen05.mma.cta_group::2 covers 256 weight rows (128 in each CTA's TMEM)
// and reads the N activation rows half from each CTA's shared memory.  Each
// CTA therefore loads only N / 2 activation rows per stage next to its
// 256 weight rows (two 128-row halves, as in the wide tiles of
// gemm_skinny.cu): per 32 KB of weights 4 KB (m <= 64) or 8 KB (m <= 128) of
// activations instead of 8 or 16, which leaves room for five stages at
// m <= 64.  The decode configuration's weight stream is bound by the bytes a
// CTA has in flight, so fewer activation bytes per stage are more weight
// bytes per SM.  The reference has no kernel for this shape (its harness only
// runs square problems, GEMMquant_sm110/src/quant_gemm_bench.cu:3038-3079);
// BASELINE config 4 names it.
//
// Work: pair p owns weight rows [512 p, 512 p + 512): CTA rank r holds rows
// 512 p + 256 h + 128 r + [0, 128) of half h.  Every pair streams its tile's
// whole K and stores its own output columns; there are no split tiles, so the
// host uses this kernel only when the tiles nearly fill the SMs (the decode
// shapes) and the stream-K kernel of gemm_skinny.cu otherwise.  The
// activations are quantised by the two kernels of gemm_skinny.cu chained
// ahead of this one with programmatic dependent launch; the producers stream
// the first weight stages and prefetch more into L2 before they wait for them.
//
// Roles (10 warps, both CTAs): warp 0 TMA producer (weights and activations
// complete on the leader's full barrier, the pair form; the scale loads on
// the leader's full barrier or the peer's own sf_full), warp 1 TMEM owner and
// in the leader the MMA issuer, warps 2..5 the epilogue (one TMEM lane
// quadrant each: lane = weight row), warps 6..9 the scale stagers
// (tcgen05.st).  No load uses cluster multicast; every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qg_codec.cuh"
#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

#ifndef QG_SKINNY_BOUNDS
#define QG_SKINNY_BOUNDS __maxnreg__(152)
#endif
// Units (32 KB of weights each) prefetched into L2 in one burst before the
// producer waits for the quantiser kernels.  Swept on one box (GB/s,
// m = 64 / 128): 4: 4706 / 4306, 8: 4734 / 4362, 16: 4754 / 4440-4458,
// 24: 4443 / 4312, 32: 4442 / 4306; a rolling lead (8 units kept ahead of
// the ring as each stage is issued): 4443 / 4052.  Again with the wider
// quantiser grid at m = 128: 8: 4690-4719 / 4551-4563, 12: 4730-4747 /
// 4543-4571, 16: 4715 / 4492-4513, 20: 4593-4606 / 4379-4383.
#ifndef QG_SKINNY_PAIR_L2_AHEAD
#define QG_SKINNY_PAIR_L2_AHEAD 12
#endif

template <int kN>
struct SkinnyPairCfg {
  static constexpr int kBM = 128;              // weight rows per CTA and half
  static constexpr int kH = 2;                 // halves per CTA
  static constexpr int kTileRows = 4 * kBM;    // weight rows per pair
  static constexpr int kBoxBytes = 128;        // one SWIZZLE_128B box: 256 fp4 of K
  static constexpr int kSfChunks = 4;          // 512-byte scale chunks (64 of K each)
  static constexpr int kMmaPerStage = kSfChunks * kH;
  static constexpr int kXRows = kN / 2;        // activation rows this CTA loads
  static constexpr int kWBox = kBM * kBoxBytes;
  static constexpr int kWBytes = kWBox * kH;
  static constexpr int kXBytes = kXRows * kBoxBytes;
  static constexpr int kSfwBytes = kSfChunks * 512 * kH;  // [half][chunk]
  static constexpr int kSfxBytes = kSfChunks * 512;       // all N rows: every CTA's MMA half reads them
  static constexpr int kAbTx = kWBytes + kXBytes;
  static constexpr int kSfTx = kSfwBytes + kSfxBytes;
  static constexpr int kStageBytes = (kAbTx + kSfTx + 1023) / 1024 * 1024;
  // Scale slot of a stage: weight scales of each half, then the activation
  // scales (4 columns per chunk each), padded to one 64-column tcgen05.st.
  static constexpr int kSfWords = 4 * kSfChunks * (kH + 1);
  static constexpr int kSfStageCols = 64;
  static constexpr int kAccCols = kH * kN;
  static constexpr int kTmemSfBase = kAccCols;
  static constexpr int kTmemCols = 512;
  // Shared memory: leave room for a quantiser CTA (1 KB static + the
  // per-CTA reserve) beside this one, so the GEMM's CTAs start at once.
  static constexpr int kSmemStages = (233472 - 3 * 1024 - 1536) / kStageBytes;
  static constexpr int kTmemStages = (kTmemCols - kTmemSfBase) / kSfStageCols;
  static constexpr int kStages0 = kSmemStages < kTmemStages ? kSmemStages : kTmemStages;
  static constexpr int kStages = kStages0 < 8 ? kStages0 : 8;
  static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
  static constexpr int kThreads = 320;
  static_assert(kN == 64 || kN == 128, "pair decode tiles take 64 or 128 activation rows");
  static_assert(kStages >= 2, "pipeline depth");
  static_assert(kSfWords <= kSfStageCols, "scale slot");
  static_assert(kTmemSfBase + kStages * kSfStageCols <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ void pair_spin_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) {
  }
}

template <int kN>
__global__ void __cluster_dims__(2, 1, 1) QG_SKINNY_BOUNDS
    gemm_skinny_pair_kernel(const __grid_constant__ SkinnyParams p) {
  using Cfg = SkinnyPairCfg<kN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* full_bar = bars;                      // leader: both CTAs' W/X + its scales
  uint64_t* sf_full = bars + Cfg::kStages;        // peer: its scales
  uint64_t* sf_ready = bars + 2 * Cfg::kStages;   // leader: 8 stager warps
  uint64_t* empty_bar = bars + 3 * Cfg::kStages;  // each CTA: the leader's MMA commit
  uint64_t* acc_full = bars + 4 * Cfg::kStages;   // each CTA
  uint64_t* drain_bar = acc_full + 1;             // leader
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int t = static_cast<int>(cluster_id_x());  // this pair's 512-row tile
  const int nkb = p.num_k_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&sf_full[s], 1);
      mbar_init(&sf_ready[s], 8);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    fence_barrier_init();
    tma_prefetch_desc(&p.tm_w);
    tma_prefetch_desc(&p.tm_x);
    tma_prefetch_desc(&p.tm_sfw);
    tma_prefetch_desc(&p.tm_sfx);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barrier inits and the TMEM allocation visible to both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Every role but the weight producer waits for the quantiser kernels here,
  // before any bounded wait starts its clock.
  if (warp != 0) griddep_wait();

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();  // weights: streamed once
      const uint64_t pol_x = l2_policy_evict_last();   // activations: read by every CTA
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      bool dep_done = false;
      int deferred = 0;
      auto stage_ptr = [&](int s) { return smem + s * Cfg::kStageBytes; };
      auto sf_bar = [&](int s) { return leader ? &full_bar[s] : &sf_full[s]; };
      // The activation part of stage s (unit kb): its scales on this CTA's
      // scale barrier, its N / 2 rows on the leader's full barrier.
      auto issue_x = [&](int s, int kb) {
        uint8_t* sx = stage_ptr(s) + Cfg::kWBytes;
        uint8_t* ssfx = sx + Cfg::kXBytes + Cfg::kSfwBytes;
        tma_load_3d(ssfx, &p.tm_sfx, sf_bar(s), 0, 0, kb * Cfg::kSfChunks, pol_x);
        tma_load_2d_pair(sx, &p.tm_x, mapa_shared(smem_u32(&full_bar[s]), 0), kb * Cfg::kBoxBytes,
                         static_cast<int>(rank) * Cfg::kXRows, pol_x);
      };
      // Before waiting for the quantiser kernels: the next units' weights
      // into L2, so the weight stream runs on while the activations are
      // quantised.
      auto prefetch_unit = [&](int kb) {
#pragma unroll
        for (int hf = 0; hf < Cfg::kH; ++hf) {
          const int rb = t * 4 + hf * 2 + static_cast<int>(rank);
          tma_prefetch_l2_3d(&p.tm_sfw, 0, rb, kb * Cfg::kSfChunks);
          tma_prefetch_l2_2d(&p.tm_w, kb * Cfg::kBoxBytes, rb * Cfg::kBM);
        }
      };
      auto release = [&](int next_kb) {
        for (int kb = next_kb; kb < nkb && kb < next_kb + QG_SKINNY_PAIR_L2_AHEAD; ++kb)
          prefetch_unit(kb);
        griddep_wait();  // the quantiser kernels have written xq / xsf
        asm volatile("fence.proxy.async.global;" ::: "memory");  // read by TMA
        for (int s = 0; s < deferred; ++s) issue_x(s, s);
        dep_done = true;
      };
      for (int kb = 0; kb < nkb; ++kb) {
        if (!dep_done && kb == Cfg::kStages) release(kb);
        if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* sw = stage_ptr(stage);
        uint8_t* ssfw = sw + Cfg::kWBytes + Cfg::kXBytes;
        if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::kAbTx + Cfg::kSfTx);
        else mbar_arrive_expect_tx(&sf_full[stage], Cfg::kSfTx);
        const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[stage]), 0);
#pragma unroll
        for (int hf = 0; hf < Cfg::kH; ++hf) {
          const int rb = t * 4 + hf * 2 + static_cast<int>(rank);  // 128-row block
          tma_load_3d(ssfw + hf * Cfg::kSfChunks * 512, &p.tm_sfw, sf_bar(stage), 0, rb,
                      kb * Cfg::kSfChunks, pol_w);
          tma_load_2d_pair(sw + hf * Cfg::kWBox, &p.tm_w, full_leader, kb * Cfg::kBoxBytes,
                           rb * Cfg::kBM, pol_w);
        }
        if (dep_done) issue_x(stage, kb);
        else ++deferred;  // stage == kb in the first lap
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == Cfg::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok && !dep_done) release(nkb);
      if (!ok) {
        // Drain: every issued stage's copies land before the CTA retires its
        // shared memory.  Scale bytes land on this CTA's barriers; W/X bytes
        // on the leader's (the peer cannot observe those, so it waits).
        uint32_t dummy = 0;
        for (int s = 0; s < Cfg::kStages; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          mbar_wait_bounded(sf_bar(s), (issued_parity >> s) & 1u, p.timeout_ns, &dummy, nullptr,
                            0);
        }
        if (!leader) pair_spin_ns(200000);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA (leader)
    if (leader && lane == 0) {
      const uint32_t idesc = make_idesc_block_scaled(2 * Cfg::kBM, kN, 1u, 0u, 0u, 0u);
      const uint64_t wdesc0 = make_smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      const uint64_t xdesc0 =
          make_smem_desc(smem_u32(smem + Cfg::kWBytes), 16, 1024, kSwizzle128B);
      constexpr uint64_t kStageDesc = Cfg::kStageBytes >> 4;
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      uint64_t wdesc = wdesc0, xdesc = xdesc0;
      uint32_t sf_col = tmem_base + Cfg::kTmemSfBase;
      for (int kb = 0; kb < nkb; ++kb) {
        // sf_ready covers the W/X bytes too: the leader's stagers arrive only
        // after its full barrier.
        if (!mbar_wait_bounded(&sf_ready[stage], phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < Cfg::kMmaPerStage; ++i) {
          // MMA i: half hf, chunk c (32-byte K step c inside the 128-byte row).
          const int hf = i / Cfg::kSfChunks, c = i % Cfg::kSfChunks;
          const uint64_t wo = static_cast<uint64_t>(hf * (Cfg::kWBox >> 4) + c * 2);
          const uint64_t xo = static_cast<uint64_t>(c * 2);
          mma_pair_mxf4nvf4(tmem_base + static_cast<uint32_t>(hf * kN), wdesc + wo, xdesc + xo,
                            idesc, sf_col + hf * 4 * Cfg::kSfChunks + c * 4,
                            sf_col + Cfg::kH * 4 * Cfg::kSfChunks + c * 4,
                            (kb | c) != 0 ? 1u : 0u);
        }
        tc_commit_pair(&empty_bar[stage], 0x3);
        if (++stage == Cfg::kStages) {
          stage = 0;
          phase ^= 1u;
          wdesc = wdesc0;
          xdesc = xdesc0;
          sf_col = tmem_base + Cfg::kTmemSfBase;
        } else {
          wdesc += kStageDesc;
          xdesc += kStageDesc;
          sf_col += Cfg::kSfStageCols;
        }
      }
      if (ok) tc_commit_pair(acc_full, 0x3);
      tc_commit_pair(drain_bar, 0x1);
      uint32_t dummy = 0;
      mbar_wait_bounded(drain_bar, 0, p.timeout_ns, &dummy, nullptr, 0);
    }
  } else if (warp >= 6) {
    // ---------------------------------------------------------------- scale stagers
    const int quad = warp % 4;
    const uint32_t t_quad = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    int stage = 0;
    uint32_t phase = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      // Leader: its full barrier (its scales and both CTAs' W/X); peer: its
      // sf_full.  The stage's TMEM slot is free then too (the producer
      // refilled the stage after the MMAs that read both had completed).
      const bool ok = mbar_wait_bounded(leader ? &full_bar[stage] : &sf_full[stage], phase,
                                        p.timeout_ns, abort_flag, p.status, kDevTimeoutMma);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint8_t* ssfw = smem + stage * Cfg::kStageBytes + Cfg::kWBytes + Cfg::kXBytes;
      const uint8_t* ssfx = ssfw + Cfg::kSfwBytes;
      uint32_t v[Cfg::kSfStageCols];
#pragma unroll
      for (int j = 0; j < Cfg::kH + 1; ++j)
#pragma unroll
        for (int c = 0; c < Cfg::kSfChunks; ++c) {
          const uint4 x = lds128((j < Cfg::kH ? ssfw + j * Cfg::kSfChunks * 512 : ssfx) + c * 512 +
                                 lane * 16);
          uint32_t* d = v + (j * Cfg::kSfChunks + c) * 4;
          d[0] = x.x;
          d[1] = x.y;
          d[2] = x.z;
          d[3] = x.w;
        }
#pragma unroll
      for (int j = Cfg::kSfWords; j < Cfg::kSfStageCols; ++j) v[j] = 0u;
      tmem_st_32x32b<Cfg::kSfStageCols>(t_quad + Cfg::kTmemSfBase + stage * Cfg::kSfStageCols, v);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&sf_ready[stage]);
        else mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&sf_ready[stage]), 0));
      }
      if (++stage == Cfg::kStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // Lane = weight row = output column n; the kN accumulator columns of a
    // half are the activation rows m.
    const int quad = warp % 4;
    const uint32_t t_quad = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const float alpha = __ldcg(p.x_ts) * (p.w_ts ? *p.w_ts : 1.0f);
    bool ok = true;
    if (lane == 0)
      ok = mbar_wait_bounded<false, 128>(acc_full, 0, p.timeout_ns, abort_flag, p.status,
                                         kDevTimeoutEpilogue);
    if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
      mbar_try_wait(acc_full, 0);
      tc_fence_after();
      const int mrows = p.m;
#pragma unroll 1
      for (int hf = 0; hf < Cfg::kH; ++hf) {
        const int n_tail = (t * 4 + hf * 2 + static_cast<int>(rank)) * Cfg::kBM + quad * 32;
        const int n = n_tail + lane;
        const bool rows16 = p.out_bf16 && p.vec_ok && n_tail + 32 <= p.n;
#pragma unroll 1
        for (int gc = 0; gc < kN / 64; ++gc) {
          uint32_t r[64];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc)
            tmem_ld_32x32b_x16(t_quad + static_cast<uint32_t>(hf * kN + gc * 64 + cc * 16),
                               *reinterpret_cast<uint32_t(*)[16]>(r + cc * 16));
          tmem_wait_ld();
          if (rows16) {
            // The stage ring is idle (every MMA that read it has completed):
            // this warp transposes its 32 columns x 64 rows through it and
            // writes C in 16-byte row pieces.
            uint8_t* tbuf = smem + quad * (64 * 64);
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 64; ++j)
              *reinterpret_cast<__nv_bfloat16*>(tbuf + j * 64 + lane * 2) =
                  __float2bfloat16_rn(__uint_as_float(r[j]) * alpha);
            __syncwarp();
            const int c16 = (lane & 3) * 16;
            uint8_t* crow = reinterpret_cast<uint8_t*>(p.c) + static_cast<int64_t>(n_tail) * 2 + c16;
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int row = it * 8 + (lane >> 2);
              const int mm = gc * 64 + row;
              const uint4 v = *reinterpret_cast<const uint4*>(tbuf + row * 64 + c16);
              if (mm < mrows)
                *reinterpret_cast<uint4*>(crow + static_cast<int64_t>(mm) * p.ldc * 2) = v;
            }
          } else if (n < p.n) {
            if (p.out_bf16) {
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.c) + n;
#pragma unroll
              for (int j = 0; j < 64; ++j)
                if (gc * 64 + j < mrows)
                  dst[static_cast<int64_t>(gc * 64 + j) * p.ldc] =
                      __float2bfloat16_rn(__uint_as_float(r[j]) * alpha);
            } else {
              float* dst = reinterpret_cast<float*>(p.c) + n;
#pragma unroll
              for (int j = 0; j < 64; ++j)
                if (gc * 64 + j < mrows)
                  dst[static_cast<int64_t>(gc * 64 + j) * p.ldc] = __uint_as_float(r[j]) * alpha;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // the leader's MMAs into both TMEMs have drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

template <int kN>
static cudaError_t launch_pair_n(const SkinnyParams& p, int grid, cudaStream_t stream) {
  using Cfg = SkinnyPairCfg<kN>;
  auto kern = gemm_skinny_pair_kernel<kN>;
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  // Programmatic dependent launch, as for gemm_skinny_kernel: the CTAs start
  // streaming weights while the quantiser kernels ahead of it still run.
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_gemm_skinny_pair(const SkinnyParams& p, int grid, cudaStream_t stream) {
  if (grid % 2 != 0) return cudaErrorInvalidValue;
  switch (skinny_mma_n(p.m)) {
    case 64: return launch_pair_n<64>(p, grid, stream);
    case 128: return launch_pair_n<128>(p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

int skinny_pair_tile_rows() { return SkinnyPairCfg<128>::kTileRows; }

}  // namespace qg
