// gemm_pair.cu -- persistent CTA-pair (cta_group::2) block-scaled GEMM.
//
// C[M,N] = alpha * A[M,K] . B[N,K]^T for NVFP4 (kind::mxf4nvf4.block16) and
// MXFP8 (kind::mxf8f6f4.block_scale), the B200 replacement for the
// reference's NVFP4 GEMM backends (CUTLASS example 72b,
// GEMMquant_sm110/build_and_run.sh:38-75; the disabled 2-SM tc6 kernel,
// GEMMsm110/include/backends/tc6_nvfp4.cuh:86-332).
//
// A cluster of two CTAs (one per SM) owns a 256 x 256 output tile at a time;
// the grid has one cluster per tile, the clusters that fit run persistently
// and take the tiles of the clusters not yet started through cluster launch
// control (clusterlaunchcontrol.try_cancel; see the tile scheduler).  Each CTA
// loads its own 128 rows of A and its own 128-row half of B; the leader CTA
// (rank 0) issues tcgen05.mma.cta_group::2, which reads A and B from both
// CTAs' shared memory and accumulates rows [0,128) in the leader's TMEM and
// rows [128,256) in the peer's.  One leader thread (warp 1) issues
// M = 256, N = 256 MMAs; a build with QG_PAIR_ISSUERS=2 splits the issue over
// warps 1 and 10 (N = 128 halves of the accumulator), which re-reads each
// CTA's A tile from shared memory per half and measured slower once the
// epilogue hands the accumulator back early (see PairCfg::kIssuers).
//
// Scale factors reach TMEM through tcgen05.st from registers, not through
// tcgen05.cp: copy instructions execute in the tensor pipe in order with the
// MMAs and cost a roughly fixed time each (12 per stage for NVFP4), which
// measured as ~45% of the kernel.  Four stager warps per CTA -- one per
// 32-lane TMEM quadrant -- read each stage's 512-byte scale chunks from shared
// memory and write the layout the MMA reads (row r at lane r%32 of every
// quadrant, column r/32, byte = scale index) for their own quadrant.
//
// Roles (both CTAs, 11 warps):
//   warp 0      TMA producer.  A/B loads complete on the LEADER's full barrier
//               (cta_group::2 form, armed by the leader with both CTAs'
//               bytes and its own scale bytes); the peer's scale loads
//               complete on its own sf_full barrier.
//   warp 1      TMEM allocation for the pair; in the leader, MMA issuer 0.
//   warp 10     in the leader, MMA issuer 1 (two-issuer builds only).
//   warps 2..5  epilogue: each CTA drains its own accumulator rows.
//   warps 6..9  scale stagers.
//   warps 11..14 (NVFP4-output kernel only) more epilogue warps.
// No TMA load uses cluster multicast.  Every wait is bounded (qg_ptx.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qg_codec.cuh"
#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

// Operand formats of the pair kernel.
constexpr int kFmtMxfp8 = 0;  // e4m3, ue8m0 per 32 K
constexpr int kFmtNvfp4 = 1;  // e2m1, ue4m3 per 16 K (+ fp32 tensor scales)
constexpr int kFmtMxfp4 = 2;  // e2m1, ue8m0 per 32 K

template <int kFmt>
struct PairCfg {
  static constexpr int kBM = 128;       // rows of A per CTA (256 per pair)
  static constexpr int kBN = 256;       // N of the pair tile
  static constexpr int kBNHalf = 128;   // rows of B each CTA loads
  static constexpr int kBKBytes = 128;  // K bytes per stage (one SWIZZLE_128B row)
#ifdef QG_PAIR_STAGES
  static constexpr int kStages = QG_PAIR_STAGES;  // A/B builds only
#else
  static constexpr int kStages = 5;
#endif
  static constexpr int kMmaPerStage = 4;
  // 512-B scale chunks (4 scales per row) along K per 128 rows per stage:
  // 256 K elements (fp4) or 128 (fp8) at 16 or 32 elements per scale.
  static constexpr int kSfChunks = kFmt == kFmtNvfp4 ? 4 : (kFmt == kFmtMxfp4 ? 2 : 1);
  static constexpr int kABytes = kBM * kBKBytes;
  static constexpr int kBBytes = kBNHalf * kBKBytes;
  // (kDiag bit 11: a diagnostic build without scale loads or their smem.)
  static constexpr int kSfaBytes = (kDiag & 2048u) ? 0 : kSfChunks * 512;
  static constexpr int kSfbBytes = (kDiag & 2048u) ? 0 : kSfChunks * 512 * 2;  // all 256 N rows in each CTA
  static constexpr int kAbTx = kABytes + kBBytes;
  static constexpr int kSfTx = kSfaBytes + kSfbBytes;
  static constexpr int kStageBytes = (kAbTx + kSfTx + 1023) / 1024 * 1024;
  // bf16 C: per epilogue warp two 64-column x 32-row staging boxes
  // (SWIZZLE_128B) for TMA stores of the output.
  static constexpr int kEpiBytes = 4 * 2 * 4096;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 512 + 1024;
  static constexpr int kSfaCols = kSfChunks * 4;
  static constexpr int kSfbCols = kSfChunks * 8;
  static constexpr int kTmemSfBase = kBN;
  // One stage's scales in TMEM: SFA then SFB columns.  Each tcgen05.st costs
  // about the same whatever its width (measured at 8192^3 NVFP4: leaving
  // out either of the two stores per stage gained ~15%), so where one slot
  // per shared-memory stage still fits beside the 256-column accumulator
  // when padded to the next store width, a stager warp writes a stage with
  // ONE store (MXFP8: 12 -> 16 columns, MXFP4: 24 -> 32; measured MXFP8 FFN
  // +10%).  NVFP4's 48 columns would pad to 64, and 5 x 64 does not fit:
  // four slots with the stagers waiting for each slot's previous MMAs
  // measured 5% slower than two stores into five 48-column slots.
  static constexpr int kTmemCols = 512;
  static constexpr int kSfCols = kSfaCols + kSfbCols;
  static constexpr int kSfColsPadded = kSfCols <= 16 ? 16 : (kSfCols <= 32 ? 32 : 64);
  static constexpr bool kOneStore = kTmemSfBase + kStages * kSfColsPadded <= kTmemCols;
  static constexpr int kTmemSfStageCols =
      (kDiag & 2048u) ? 16 : (kOneStore ? kSfColsPadded : kSfCols);
  static_assert(kTmemSfBase + kStages * kTmemSfStageCols <= kTmemCols, "TMEM budget");
  // TMEM column of a slot's SFA and SFB (SFB right after SFA).
  static constexpr int kSfaStep = kTmemSfStageCols;
  static constexpr int kSfbBase = kTmemSfBase + kSfaCols;
  static constexpr int kSfbStep = kTmemSfStageCols;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  // One MMA issuer with N = 256 MMAs by default: each CTA's tensor core
  // then reads its A tile once per K step.  Two issuers (N = 128 halves,
  // QG_PAIR_ISSUERS=2 at build time) read it twice; measured on one box with
  // the eight-warp epilogue, one issuer is faster in every format (NVFP4
  // 8192^3 4693 -> 4990 TF/s, MXFP4 5156 -> 5235, MXFP8 2424 -> 2450).
#ifdef QG_PAIR_ISSUERS
  static constexpr int kIssuers = QG_PAIR_ISSUERS;
#else
  static constexpr int kIssuers = 1;
#endif
  static constexpr int kIssueN = kBN / kIssuers;
  static constexpr int kThreads = 320 + 32 * (kIssuers - 1);
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

// Diagnostic timeline (kDiag bit 9; the output buffer is overwritten): the
// roles of the first pair's CTAs write %globaltimer stamps of their waits
// into C, 2048 slots per event kind, so a host script can see which wait
// bounds the pipeline.  Compiled out of shipped builds.
constexpr bool kTracePair = (kDiag & 512u) != 0;
__device__ __forceinline__ void trace_pair(const GemmParams& p, bool on, int kind, int slot) {
  if (kTracePair && on && slot < 2048)
    reinterpret_cast<unsigned long long*>(p.c)[kind * 2048 + slot] = globaltimer_ns();
}

// One stage's scales of this warp's TMEM quadrant: SFA chunks (4 columns
// each, the 16-byte row r of a chunk holds rows r, r+32, r+64, r+96) and the
// two 128-row SFB blocks per chunk (8 columns per chunk).
template <int kFmt>
__device__ __forceinline__ void stage_scales(const uint8_t* ssfa, const uint8_t* ssfb,
                                             uint32_t t_slot, int lane) {
  using Cfg = PairCfg<kFmt>;
  // SFA columns [0, kSfaCols), SFB columns [kSfaCols, kSfCols), padding.
  uint32_t v[Cfg::kOneStore ? Cfg::kTmemSfStageCols : Cfg::kSfCols];
#pragma unroll
  for (int i = Cfg::kSfCols; i < (Cfg::kOneStore ? Cfg::kTmemSfStageCols : Cfg::kSfCols); ++i)
    v[i] = 0u;
  uint32_t* a = v;
  uint32_t* b = v + Cfg::kSfaCols;
#pragma unroll
  for (int c = 0; c < Cfg::kSfChunks; ++c) {
    const uint4 x = lds128(ssfa + c * 512 + lane * 16);
    a[4 * c] = x.x;
    a[4 * c + 1] = x.y;
    a[4 * c + 2] = x.z;
    a[4 * c + 3] = x.w;
    const uint4 w0 = lds128(ssfb + (c * 2) * 512 + lane * 16);
    const uint4 w1 = lds128(ssfb + (c * 2 + 1) * 512 + lane * 16);
    if (Cfg::kIssuers == 2) {
      // Issuer 0's MMA B rows are tile rows 0-63 | 128-191, issuer 1's
      // 64-127 | 192-255 (each CTA contributes half of an MMA's N): column
      // r/32 of a 128-row block holds rows 32*col.., so the halves take
      // columns {0,1} and {2,3} of both blocks.
      b[8 * c] = w0.x;
      b[8 * c + 1] = w0.y;
      b[8 * c + 2] = w1.x;
      b[8 * c + 3] = w1.y;
      b[8 * c + 4] = w0.z;
      b[8 * c + 5] = w0.w;
      b[8 * c + 6] = w1.z;
      b[8 * c + 7] = w1.w;
    } else {
      b[8 * c] = w0.x;
      b[8 * c + 1] = w0.y;
      b[8 * c + 2] = w0.z;
      b[8 * c + 3] = w0.w;
      b[8 * c + 4] = w1.x;
      b[8 * c + 5] = w1.y;
      b[8 * c + 6] = w1.z;
      b[8 * c + 7] = w1.w;
    }
  }
  if constexpr (Cfg::kOneStore) {
    tmem_st_32x32b<Cfg::kTmemSfStageCols>(t_slot, v);
  } else {
    tmem_st_32x32b<Cfg::kSfaCols>(t_slot, *reinterpret_cast<uint32_t(*)[Cfg::kSfaCols]>(a));
    tmem_st_32x32b<Cfg::kSfbCols>(t_slot + Cfg::kSfaCols,
                                  *reinterpret_cast<uint32_t(*)[Cfg::kSfbCols]>(b));
  }
}

// Tile order: groups of kGroupM m-tiles, n-tiles outer within a group, so
// the pairs working at one time share a few A slices and B slices in L2
// (a wave of 74 pairs covers kGroupM m-tiles x ~5 n-tiles instead of every
// m-tile of one column, which re-read all of A from HBM once per wave when A
// outgrew L2: 16384 x 8192 A is 67 MB of values next to a streaming output).
#ifdef QG_PAIR_GROUP_M
constexpr int kGroupM = QG_PAIR_GROUP_M;  // A/B builds only
#else
constexpr int kGroupM = 16;
#endif
__device__ __forceinline__ void tile_coords(int tile, int num_m_tiles, int num_n_tiles, int& mt,
                                            int& nt) {
  const int per_group = kGroupM * num_n_tiles;
  const int g = tile / per_group, r = tile - g * per_group;
  const int m0 = g * kGroupM;
  const int gm = num_m_tiles - m0 < kGroupM ? num_m_tiles - m0 : kGroupM;
  mt = m0 + r % gm;
  nt = r / gm;
}

// kOut: 0 fp32 C, 1 bf16 C, 2 NVFP4 output (values + e4m3 block scales,
// requantised in the epilogue as the reference's tc6 store_tile does,
// GEMMsm110/include/backends/tc6_nvfp4.cuh:460-503).
// Threads per CTA: 11 warps; the NVFP4-output epilogue (kOut 2) and the
// bf16 TMA-store epilogue (kOut 3) add four more epilogue warps (11..14, one
// per TMEM lane quadrant).
template <int kOut>
constexpr int pair_threads() {
  return kOut >= 2 ? 480 : 352;
}

// ------------------------------------------------------------------ tile scheduler
// The grid holds one CTA pair per output tile; the pairs that fit run
// persistently and take the tiles of pairs not yet started with cluster
// launch control (clusterlaunchcontrol.try_cancel): the hardware cancels a
// pending cluster and hands its index to the caller, so the work is spread
// over whatever SMs are running it, with no static assignment.  The leader's
// producer thread is the scheduler.  It asks for the next tile while the
// current tile's loads stream and publishes each tile index (-1: no work
// left) through a small ring in both CTAs' shared memory: the index word
// plus a full barrier per slot in each CTA (the peer's written over the
// cluster's shared-memory window), and one empty barrier per slot in the
// leader that every consumer (both CTAs' producer / issuer / stager /
// epilogue warps) arrives on once it has read the index.
constexpr int kTileRing = 2;

// Consumers of a ring slot: the leader's issuer thread(s), 4 stager warps
// and the epilogue warps of each CTA, and the peer's producer thread.
template <int kOut>
__host__ __device__ constexpr int tile_consumers(int issuers) {
  return issuers + 1 + 2 * (4 + (kOut >= 2 ? 8 : 4));
}

struct TileRing {
  volatile int32_t* ids;  // [kTileRing] this CTA's copy of each slot's tile index
  uint64_t* full;         // [kTileRing] this CTA
  uint64_t* empty;        // [kTileRing] leader's
  bool leader;
  int slot = 0;
  uint32_t phase = 0;

  // Consumer: the next tile index (-1 when the work is done, -2 when a wait
  // timed out).  One thread of the consuming warp calls it.
  __device__ int next(const GemmParams& p, volatile uint32_t* abort_flag) {
    // The leader's slots are written locally (release.cta arrive), the
    // peer's over the cluster window (release.cluster arrive).
    const bool ok = leader ? mbar_wait_bounded(&full[slot], phase, p.timeout_ns, abort_flag,
                                               p.status, kDevTimeoutMma)
                           : mbar_wait_bounded<true>(&full[slot], phase, p.timeout_ns,
                                                     abort_flag, p.status, kDevTimeoutMma);
    if (!ok) return -2;
    // Acquire load, then a relaxed arrive: the arrive that frees the slot
    // cannot pass the read, and it need not wait for this warp's earlier
    // writes (a release-scoped arrive would, e.g. for the epilogue's
    // stores, on the tile boundary's critical path).
    const int t = ld_acquire_shared_s32(&ids[slot]);
    if (leader) mbar_arrive_relaxed(&empty[slot]);
    else mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&empty[slot]), 0));
    if (++slot == kTileRing) {
      slot = 0;
      phase ^= 1u;
    }
    return t;
  }
  // Warp-wide form: lane 0 takes the index, every lane gets it.
  __device__ int next_warp(const GemmParams& p, volatile uint32_t* abort_flag, int lane) {
    int t = 0;
    if (lane == 0) t = next(p, abort_flag);
    t = __shfl_sync(0xffffffffu, t, 0);
    if (lane != 0 && ++slot == kTileRing) {  // keep every lane's cursor in step
      slot = 0;
      phase ^= 1u;
    }
    return t;
  }
  // Scheduler (leader's producer thread): publish `t` into the next slot of
  // both CTAs once every consumer has read the slot's previous index.
  __device__ bool publish(const GemmParams& p, volatile uint32_t* abort_flag, int t) {
    if (!mbar_wait_bounded(&empty[slot], phase ^ 1u, p.timeout_ns, abort_flag, p.status,
                           kDevTimeoutProducer))
      return false;
    ids[slot] = t;
    st_shared_cluster_u32(mapa_shared(smem_u32(const_cast<int32_t*>(&ids[slot])), 1),
                          static_cast<uint32_t>(t));
    mbar_arrive(&full[slot]);
    mbar_arrive_cluster(mapa_shared(smem_u32(&full[slot]), 1));  // release: the word first
    if (++slot == kTileRing) {
      slot = 0;
      phase ^= 1u;
    }
    return true;
  }
};

template <int kFmt, int kOut>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads<kOut>(), 1)
    gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = PairCfg<kFmt>;
  constexpr bool kFp4 = kFmt != kFmtMxfp8;
  constexpr bool kOutBf16 = kOut == 1 || kOut == 3;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* epi_smem = smem + Cfg::kStages * Cfg::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + Cfg::kEpiBytes);
  uint64_t* full_bar = bars;                        // leader: A/B bytes of both CTAs
  uint64_t* sf_full = bars + Cfg::kStages;          // each CTA: its scale bytes
  uint64_t* sf_ready = bars + 2 * Cfg::kStages;     // leader: 8 stager warps
  uint64_t* empty_bar = bars + 3 * Cfg::kStages;    // each CTA
  uint64_t* acc_full = bars + 4 * Cfg::kStages;     // each CTA
  uint64_t* acc_empty = acc_full + 1;               // leader: [kIssuers], 8 epilogue warps
  uint64_t* drain_bar = acc_full + 3;               // leader: [kIssuers]
  uint64_t* tile_full = acc_full + 5;               // each CTA: [kTileRing], the scheduler
  uint64_t* tile_empty = tile_full + kTileRing;      // leader: [kTileRing], every consumer
  uint64_t* clc_bar = tile_empty + kTileRing;        // leader: the cancel response
  uint8_t* clc_resp = reinterpret_cast<uint8_t*>(  // 16 B, 16-byte aligned
      (reinterpret_cast<uintptr_t>(clc_bar + 1) + 15) & ~static_cast<uintptr_t>(15));
  volatile int32_t* tile_ids = reinterpret_cast<volatile int32_t*>(clc_resp + 16);  // [kTileRing]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(clc_resp + 16 + 4 * kTileRing);
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
      mbar_init(&empty_bar[s], Cfg::kIssuers);
    }
    mbar_init(acc_full, Cfg::kIssuers);
    for (int i = 0; i < Cfg::kIssuers; ++i) mbar_init(&acc_empty[i], kOut >= 2 ? 16 : 8);
    for (int i = 0; i < Cfg::kIssuers; ++i) mbar_init(&drain_bar[i], 1);
    for (int i = 0; i < kTileRing; ++i) {
      mbar_init(&tile_full[i], 1);
      mbar_init(&tile_empty[i], tile_consumers<kOut>(Cfg::kIssuers));
    }
    mbar_init(clc_bar, 1);
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
  (void)num_tiles;
  (void)npairs;
  // Every role of both CTAs takes the cluster's tiles from the tile ring:
  // the first is the cluster's own index, later ones come from the
  // leader's producer through cluster launch control (see TileRing).
  TileRing ring{tile_ids, tile_full, tile_empty, leader};

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      // B tiles (and their scales): within a group of kGroupM m-tiles the
      // pairs working at one time share a B tile once, A slices are reused
      // across the group's n-tiles.  A/B builds may mark B evict-first.
#ifdef QG_PAIR_B_EVICT_FIRST
      const uint64_t pol_b = l2_policy_evict_first();
#else
      const uint64_t pol_b = pol;
#endif
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      bool clc_pending = false;
      uint32_t clc_phase = 0;
      int stage = 0, kb = 0, g = 0;
      uint32_t phase = 0;
      int mt = 0, nt = 0;
      const bool skip_loads = (kDiag & 4u) != 0;
      // The leader's producer schedules: the cluster's own tile first.
      int tile = leader ? pair : ring.next(p, abort_flag);
      int next_tile = -1;
      // The cancelled cluster's tile (its first CTA's index / 2), or -1,
      // published to every consumer of both CTAs.
      auto publish_next = [&]() -> bool {
        if (!mbar_wait_bounded(clc_bar, clc_phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutProducer))
          return false;
        clc_pending = false;
        clc_phase ^= 1u;
        const int x = clc_first_ctaid_x(clc_resp);
        next_tile = x < 0 ? -1 : x / 2;
        return ring.publish(p, abort_flag, next_tile);
      };
      if (leader) ok = ring.publish(p, abort_flag, tile);
      if (tile < 0) ok = ok && tile == -1;
      while (ok && tile >= 0) {
        tile_coords(tile, p.num_m_tiles, p.num_n_tiles, mt, nt);
        if (leader) {
          // Ask for the next tile now; the answer is read after this tile's
          // loads are issued.
          mbar_arrive_expect_tx(clc_bar, 16);
          clc_try_cancel(clc_resp, clc_bar);
          clc_pending = true;
        }
        for (kb = 0; kb < nkb; ++kb, ++g) {
          if (g > 0 && ++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
          }
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          trace_pair(p, pair == 0, leader ? 0 : 8, g);
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          uint8_t* ssfa = sb + Cfg::kBBytes;
          uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
          if (skip_loads) {
            mbar_arrive(leader ? &full_bar[stage] : &sf_full[stage]);
            continue;
          }
          const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[stage]), 0);
          // The leader's scales complete on its full barrier with both CTAs'
          // A/B bytes (its stagers then wait once per stage, and their arrival
          // on sf_ready also tells the issuer that A/B have landed); the
          // peer's scales complete on its own sf_full.  Scales go first: they
          // are small and land early.
          uint64_t* sf_bar = leader ? &full_bar[stage] : &sf_full[stage];
          // Diagnostic builds may leave out the B (kDiag bit 7) or the SFB
          // (bit 8) loads to weigh the load path; shipped builds load all.
          constexpr bool kLoadB = (kDiag & 128u) == 0;
          constexpr bool kLoadSfb = (kDiag & 256u) == 0 && Cfg::kSfbBytes > 0;
          constexpr uint32_t kSfTxHere = Cfg::kSfaBytes + (kLoadSfb ? Cfg::kSfbBytes : 0);
          constexpr uint32_t kAbTxHere = Cfg::kABytes + (kLoadB ? Cfg::kBBytes : 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * kAbTxHere + kSfTxHere);
          else mbar_arrive_expect_tx(&sf_full[stage], kSfTxHere);
          if (Cfg::kSfaBytes > 0)
            tma_load_3d(ssfa, &p.tm_sfa, sf_bar, 0, mt * 2 + static_cast<int>(rank),
                        kb * Cfg::kSfChunks, pol);
          if (kLoadSfb) tma_load_3d(ssfb, &p.tm_sfb, sf_bar, 0, nt * 2, kb * Cfg::kSfChunks, pol_b);
          tma_load_2d_pair(sa, &p.tm_a, full_leader, kb * Cfg::kBKBytes,
                           mt * 2 * Cfg::kBM + static_cast<int>(rank) * Cfg::kBM, pol);
          if (kLoadB)
            tma_load_2d_pair(sb, &p.tm_b, full_leader, kb * Cfg::kBKBytes,
                             nt * Cfg::kBN + static_cast<int>(rank) * Cfg::kBNHalf, pol_b);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        }
        if (!ok) break;
        if (leader) {
          // The next tile, published once this tile's loads are issued
          // (publishing it a few stages earlier measured 1-4% slower).
          if (!publish_next()) {
            ok = false;
            break;
          }
          tile = next_tile;
        } else {
          tile = ring.next(p, abort_flag);
          if (tile == -2) ok = false;
        }
      }
      if (clc_pending) {
        // A cancel request still in flight writes this CTA's shared memory:
        // let it land before the CTA exits.
        uint32_t dummy = 0;
        mbar_wait_bounded(clc_bar, clc_phase, p.timeout_ns, &dummy, nullptr, 0);
      }
      if (!ok) {
        // Drain: every issued stage's copies land before the CTA retires its
        // shared memory.  Scale bytes land on this CTA's barriers; A/B bytes
        // on the leader's (the peer cannot observe those, so it waits).
        uint32_t dummy = 0;
        for (int s = 0; s < Cfg::kStages; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          mbar_wait_bounded(leader ? &full_bar[s] : &sf_full[s], (issued_parity >> s) & 1u,
                            p.timeout_ns, &dummy, nullptr, 0);
        }
        if (!leader) spin_ns(200000);
      }
    }
  } else if (warp == 1 || warp == 10) {
    // ---------------------------------------------------------------- MMA
    // Issuer h (warp 1: h = 0, warp 10: h = 1) accumulates output columns of
    // its N half into TMEM columns [h * kIssueN, (h + 1) * kIssueN).  The
    // issue loop is the pipeline's serial path (one thread per issuer):
    // stage, phase, descriptors and scale columns are stepped by constants
    // and the diagnostic switches are read once.
    const int h = warp == 1 ? 0 : 1;
    if (leader && lane == 0 && h < Cfg::kIssuers) {
      const uint32_t idesc_base =
          kFp4 ? make_idesc_block_scaled(2 * Cfg::kBM, Cfg::kIssueN, 1u,
                                         kFmt == kFmtMxfp4 ? 1u : 0u, 0u, 0u)
               : make_idesc_block_scaled(2 * Cfg::kBM, Cfg::kIssueN, 0u, 1u, 0u, 0u);
      const bool skip_mma = (kDiag & 2u) != 0;
      // B rows [h * kIssueN / 2, +kIssueN / 2) of each CTA's 128-row half.
      const uint64_t adesc0 = make_smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      const uint64_t bdesc0 =
          adesc0 + ((Cfg::kABytes + h * (Cfg::kIssueN / 2) * Cfg::kBKBytes) >> 4);
      constexpr uint64_t kStageDesc = Cfg::kStageBytes >> 4;
      const uint32_t sf0 = tmem_base + Cfg::kTmemSfBase;
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(h * Cfg::kIssueN);
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      uint64_t adesc = adesc0, bdesc = bdesc0;
      uint32_t sfa_col = sf0;
      const uint32_t sfb0 = tmem_base + Cfg::kSfbBase;
      uint32_t sfb_col = sfb0;
      for (int it = 0; ok; ++it) {
        const int tile = ring.next(p, abort_flag);
        if (tile < 0) {
          ok = tile == -1;
          break;
        }
        if (!mbar_wait_bounded(&acc_empty[h], (it & 1) ^ 1u, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma)) {
          ok = false;
          break;
        }
        trace_pair(p, pair == 0, 7, it);
        tc_fence_after();
        uint32_t acc = 0;
        for (int kb = 0; kb < nkb; ++kb) {
          // sf_ready covers the A/B bytes too: the leader's stagers arrive
          // only after full_bar.
          trace_pair(p, pair == 0, 20, it * nkb + kb);
          if (!mbar_wait_bounded(&sf_ready[stage], phase, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutMma)) {
            ok = false;
            break;
          }
          trace_pair(p, pair == 0, 3, it * nkb + kb);
          tc_fence_after();
          if (!skip_mma) {
#pragma unroll
            for (int j = 0; j < Cfg::kMmaPerStage; ++j) {
              const uint64_t koff = static_cast<uint64_t>(j * 2);  // +32 B of K
              if (kFmt == kFmtMxfp4) {
                // Chunk j/2 holds this MMA's scales; ids 0 / 2 pick the pair.
                const uint32_t sid = static_cast<uint32_t>((j & 1) * 2);
                mma_pair_mxf4(d_tmem, adesc + koff, bdesc + koff,
                              idesc_base | (sid << 29) | (sid << 4), sfa_col + (j / 2) * 4,
                              sfb_col + (j / 2) * 8 + h * 4, acc);
              } else if (kFp4) {
                mma_pair_mxf4nvf4(d_tmem, adesc + koff, bdesc + koff, idesc_base,
                                  sfa_col + j * 4, sfb_col + j * 8 + h * 4, acc);
              } else {
                const uint32_t idesc = idesc_base | (static_cast<uint32_t>(j) << 29) |
                                       (static_cast<uint32_t>(j) << 4);
                mma_pair_mxf8f6f4(d_tmem, adesc + koff, bdesc + koff, idesc, sfa_col,
                                  sfb_col + h * 4, acc);
              }
              acc = 1;
            }
          }
          trace_pair(p, pair == 0, 19, it * nkb + kb);
          tc_commit_pair(&empty_bar[stage], 0x3);
          trace_pair(p, pair == 0, 4, it * nkb + kb);
          if (++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
            adesc = adesc0;
            bdesc = bdesc0;
            sfa_col = sf0;
            sfb_col = sfb0;
          } else {
            adesc += kStageDesc;
            bdesc += kStageDesc;
            sfa_col += Cfg::kSfaStep;
            sfb_col += Cfg::kSfbStep;
          }
        }
        if (ok) tc_commit_pair(acc_full, 0x3);
      }
      tc_commit_pair(&drain_bar[h], 0x1);
      uint32_t dummy = 0;
      mbar_wait_bounded(&drain_bar[h], 0, p.timeout_ns, &dummy, nullptr, 0);
    }
  } else if (warp >= 6 && warp <= 9) {
    // ---------------------------------------------------------------- scale stagers
    const int quad = warp % 4;
    const uint32_t t_quad = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const bool no_wait = (kDiag & 32u) != 0, skip_st = (kDiag & 1u) != 0;
    int stage = 0;
    uint32_t phase = 0;
    bool run = true;
    for (int g = 0; run;) {
      const int tile = ring.next_warp(p, abort_flag, lane);
      if (tile < 0) break;
      for (int kb = 0; kb < nkb; ++kb, ++g) {
        if (g > 0 && ++stage == Cfg::kStages) {
          stage = 0;
          phase ^= 1u;
        }
        // Every lane polls (and so acquires) the stage barrier itself: one
        // wait per stage on the stager's serial path.  Leader: the full
        // barrier (its scales and both CTAs' A/B); peer: its sf_full.  The
        // stage's TMEM slot is free then too (the producer refilled the
        // stage after the MMAs that read both had completed).
        bool ok = no_wait || mbar_wait_bounded(leader ? &full_bar[stage] : &sf_full[stage], phase,
                                               p.timeout_ns, abort_flag, p.status, kDevTimeoutMma);
        if (!__all_sync(0xffffffffu, ok)) {
          run = false;
          break;
        }
        trace_pair(p, pair == 0 && warp == 6 && lane == 0, leader ? 1 : 9, g);
        const uint8_t* ssfa = smem + stage * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes;
        const uint8_t* ssfb = ssfa + Cfg::kSfaBytes;
        const uint32_t sfa_col = Cfg::kTmemSfBase + stage * Cfg::kTmemSfStageCols;
        if (!skip_st) {
          stage_scales<kFmt>(ssfa, ssfb, t_quad + sfa_col, lane);
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (leader) {
          if (lane == 0) mbar_arrive(&sf_ready[stage]);
        } else if (lane == 0) {
          // A release-scoped arrive at cluster scope costs ~1 us here and
          // serialises the stagers (measured: 2.2 vs 4.1 PF/s).  The relaxed
          // arrive is enough: tcgen05.wait::st has already completed the TMEM
          // writes and tcgen05.fence::before_thread_sync orders them before it.
          mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&sf_ready[stage]), 0));
        }
        trace_pair(p, pair == 0 && warp == 6 && lane == 0, leader ? 2 : 10, g);
        trace_pair(p, pair == 0 && lane == 0, 11 + (warp - 6) + (leader ? 0 : 4), g);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp % 4;
    // acc_empty[h] (leader) is released as soon as this warp has read issuer
    // h's TMEM columns, so issuer 0 starts the next tile while the second
    // half is still being read.  Relaxed remote arrive: tcgen05.wait::ld has
    // completed the reads and fence::before_thread_sync orders them first.
    const uint32_t acc_empty_leader0 = mapa_shared(smem_u32(&acc_empty[0]), 0);
    const uint32_t acc_empty_leader1 = mapa_shared(smem_u32(&acc_empty[Cfg::kIssuers - 1]), 0);
    float alpha = 1.0f;
    if (p.a_ts) alpha *= *p.a_ts;
    if (p.b_ts) alpha *= *p.b_ts;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    // 64-column blocks: with two issuers TMEM block 1 holds output block 2
    // and block 2 output block 1 (issuer h's MMA N rows are h*64.. of each
    // CTA's half); the map is its own inverse.
    auto tmem_block = [](int b) { return Cfg::kIssuers == 2 && (b == 1 || b == 2) ? 3 - b : b; };
    // NVFP4 output: 1 / tensor scale (IEEE division, as the reference's host
    // quantizer forms it) and the running amax of this lane's outputs.
    float rq_inv_ts = 1.0f, rq_max = 0.0f;
    if constexpr (kOut == 2) rq_inv_ts = __fdiv_rn(1.0f, p.rq_ts ? *p.rq_ts : 1.0f);
    for (int it = 0;; ++it) {
      const int tile = ring.next_warp(p, abort_flag, lane);
      if (tile < 0) break;
      int mt, nt;
      tile_coords(tile, p.num_m_tiles, p.num_n_tiles, mt, nt);
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded<false, 32>(acc_full, it & 1, p.timeout_ns, abort_flag, p.status,
                                          kDevTimeoutEpilogue);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(acc_full, it & 1);
      tc_fence_after();
      const int row = mt * 2 * Cfg::kBM + static_cast<int>(rank) * Cfg::kBM + quad * 32 + lane;
      const bool row_ok = row < p.m && !(kDiag & 8u);
      const int n0 = nt * Cfg::kBN;
      if constexpr (kOut == 2) {
        // NVFP4 output.  Each lane owns one output row, so a 16-column block
        // (one e4m3 scale) lies in one thread's registers: the block amax
        // needs no shuffles.  The element values are alpha * acc, the same
        // fp32 numbers the fp32-output GEMM stores, quantised with the
        // make_nvfp4_reference steps
        // (GEMMsm110/include/requant/nvfp4_reference.cuh:76-112) under the
        // caller's tensor scale.  Two warps per TMEM lane quadrant (warps 2-5
        // and 11-14) split the columns: for each issuer's 128-column half a
        // warp loads its 64 columns, hands the half back at once (the next
        // tile's MMAs start while this tile is requantised), then encodes.
        const int sub = warp >= 11 ? 1 : 0;
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          const int tb = 2 * h + sub;
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(t_row + tb * 64, r0);
          tmem_ld_32x32b_x32(t_row + tb * 64 + 32, r1);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          // Two issuers: each 128-column half goes back on its own barrier;
          // one issuer: the accumulator goes back once both halves are read.
          if (lane == 0 && (Cfg::kIssuers == 2 || h == 1))
            mbar_arrive_cluster_relaxed(h ? acc_empty_leader1 : acc_empty_leader0);
          const int col0 = n0 + tmem_block(tb) * 64;
          if (!row_ok || col0 >= p.n) continue;
          uint32_t w[8];
          uint32_t sbits[4];
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t* src = g < 2 ? r0 + g * 16 : r1 + (g - 2) * 16;
            float v[16];
            float bmax = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              v[i] = __fmul_rn(__uint_as_float(src[i]), alpha);
              bmax = fmaxf(bmax, fabsf(v[i]));
            }
            if (col0 + 16 * g < p.n) rq_max = fmaxf(rq_max, bmax);
            sbits[g] = nvfp4_encode_block_cvt(v, bmax, rq_inv_ts, w[2 * g], w[2 * g + 1]);
            if (p.rq_layout == 0) {
              // REF_LINEAR: element 2i in the high nibble (pack_fp4.cuh:11-15).
              w[2 * g] = ((w[2 * g] & 0x0f0f0f0fu) << 4) | ((w[2 * g] >> 4) & 0x0f0f0f0fu);
              w[2 * g + 1] =
                  ((w[2 * g + 1] & 0x0f0f0f0fu) << 4) | ((w[2 * g + 1] >> 4) & 0x0f0f0f0fu);
            }
          }
          const int64_t e0 = static_cast<int64_t>(row) * p.n + col0;
          const bool full = col0 + 64 <= p.n;
          if (full && (p.n % 32) == 0) {
            uint4* dst = reinterpret_cast<uint4*>(p.rq_q + e0 / 2);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          } else {
#pragma unroll
            for (int g = 0; g < 4; ++g)
              if (col0 + 16 * g < p.n)
                reinterpret_cast<uint2*>(p.rq_q + e0 / 2)[g] = make_uint2(w[2 * g], w[2 * g + 1]);
          }
          int64_t so;
          bool word;
          if (p.rq_layout == 0) {
            so = e0 / 16;
            word = full && (p.n % 64) == 0;
          } else {
            so = mma_scale_offset(row, col0 / 16, p.rq_row_blocks, p.rq_sf_blocks, p.rq_layout);
            word = full;
          }
          if (word) {
            *reinterpret_cast<uint32_t*>(p.rq_sf + so) =
                sbits[0] | (sbits[1] << 8) | (sbits[2] << 16) | (sbits[3] << 24);
          } else {
#pragma unroll
            for (int g = 0; g < 4; ++g)
              if (col0 + 16 * g < p.n) p.rq_sf[so + g] = static_cast<uint8_t>(sbits[g]);
          }
        }
      } else if constexpr (kOut == 3) {
        // bf16 through TMA stores with eight epilogue warps (2-5, 11-14; two
        // per TMEM lane quadrant); a warp owns TMEM blocks `sub` and
        // 2 + `sub` (64 columns each) of its quadrant.  With one issuer the
        // next tile's MMAs need the whole accumulator back, so a warp reads
        // both blocks before any TMA store (the first converted to bf16 and
        // staged in the warp's swizzled 4 KB box while the second is read),
        // hands the accumulator back, and only then issues the box stores:
        // the next tile's MMAs start while this tile's output is written.
        const int sub = warp >= 11 ? 1 : 0;
        const int row0 = mt * 2 * Cfg::kBM + static_cast<int>(rank) * Cfg::kBM + quad * 32;
        uint8_t* box = epi_smem + (quad * 2 + sub) * 4096;
        trace_pair(p, pair == 0 && leader && warp == 2 && lane == 0, 5, it);
        auto convert = [&](const uint32_t(&r0)[32], const uint32_t(&r1)[32], uint4(&v)[8]) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t* src = c < 4 ? r0 + c * 8 : r1 + (c - 4) * 8;
            v[c] = make_uint4(
                bf16x2_bits(__uint_as_float(src[0]) * alpha, __uint_as_float(src[1]) * alpha),
                bf16x2_bits(__uint_as_float(src[2]) * alpha, __uint_as_float(src[3]) * alpha),
                bf16x2_bits(__uint_as_float(src[4]) * alpha, __uint_as_float(src[5]) * alpha),
                bf16x2_bits(__uint_as_float(src[6]) * alpha, __uint_as_float(src[7]) * alpha));
          }
        };
        auto write_box = [&](const uint4(&v)[8]) {
          if (lane == 0) tma_store_wait_read<0>();  // the box's previous store has read it
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(box + lane * 128 + ((c ^ (lane & 7)) * 16)) = v[c];
          fence_proxy_async_smem();
          __syncwarp();
        };
        auto store_box = [&](int tb) {
          if (lane == 0 && !(kDiag & 8u)) {
            for (int d = 0; d < p.n_out; ++d)
              tma_store_2d(&p.tm_out[d], box, n0 + tmem_block(tb) * 64, row0);
            tma_store_commit();
          }
        };
        if constexpr (Cfg::kIssuers == 1) {
          {
            uint32_t r0[32], r1[32];
            uint4 v[8];
            tmem_ld_32x32b_x32(t_row + sub * 64, r0);
            tmem_ld_32x32b_x32(t_row + sub * 64 + 32, r1);
            tmem_wait_ld();
            convert(r0, r1, v);
            write_box(v);  // the previous tile's last store read this box long ago
          }
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(t_row + (2 + sub) * 64, r0);
          tmem_ld_32x32b_x32(t_row + (2 + sub) * 64 + 32, r1);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster_relaxed(acc_empty_leader0);
          trace_pair(p, pair == 0 && leader && warp == 2 && lane == 0, 6, it);
          store_box(sub);
          uint4 v[8];
          convert(r0, r1, v);
          write_box(v);
          store_box(2 + sub);
        } else {
          // Two issuers: each 128-column half goes back on its own barrier
          // as soon as it has been read.
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            const int tb = 2 * h + sub;
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(t_row + tb * 64, r0);
            tmem_ld_32x32b_x32(t_row + tb * 64 + 32, r1);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(h ? acc_empty_leader1 : acc_empty_leader0);
            uint4 v[8];
            convert(r0, r1, v);
            write_box(v);
            store_box(tb);
          }
        }
      } else if (Cfg::kEpiBytes > 0 && kOutBf16 && p.n_out > 0) {
        // TMEM -> registers -> bf16 in a swizzled shared-memory box -> TMA
        // store (coalesced, asynchronous, clipped at the matrix edge) to each
        // destination; for the fused gather the peers' copies cross NVLink
        // while the next tiles are computed.  One 64-column TMEM block per
        // box; two boxes alternate.
        const int row0 = mt * 2 * Cfg::kBM + static_cast<int>(rank) * Cfg::kBM + quad * 32;
        uint8_t* ebuf = epi_smem + quad * 8192;
#pragma unroll
        for (int q = 0; q < Cfg::kBN / 64; ++q) {
          uint8_t* box = ebuf + (q & 1) * 4096;
          if ((q & 1) == 0) {
            if (lane == 0) tma_store_wait_read<0>();  // both boxes read by earlier stores
            __syncwarp();
          }
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(t_row + q * 64, r0);
          tmem_ld_32x32b_x32(t_row + q * 64 + 32, r1);
          tmem_wait_ld();
          if ((Cfg::kIssuers == 2 && q == Cfg::kBN / 128 - 1) || q == Cfg::kBN / 64 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
              mbar_arrive_cluster_relaxed(q == Cfg::kBN / 64 - 1 ? acc_empty_leader1
                                                                 : acc_empty_leader0);
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t* src = c < 4 ? r0 + c * 8 : r1 + (c - 4) * 8;
            const uint4 v = make_uint4(
                bf16x2_bits(__uint_as_float(src[0]) * alpha, __uint_as_float(src[1]) * alpha),
                bf16x2_bits(__uint_as_float(src[2]) * alpha, __uint_as_float(src[3]) * alpha),
                bf16x2_bits(__uint_as_float(src[4]) * alpha, __uint_as_float(src[5]) * alpha),
                bf16x2_bits(__uint_as_float(src[6]) * alpha, __uint_as_float(src[7]) * alpha));
            *reinterpret_cast<uint4*>(box + lane * 128 + ((c ^ (lane & 7)) * 16)) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && !(kDiag & 8u)) {
            for (int d = 0; d < p.n_out; ++d)
              tma_store_2d(&p.tm_out[d], box, n0 + tmem_block(q) * 64, row0);
            tma_store_commit();
          }
        }
      } else {
        // fp32 output, or bf16 C that TMA cannot store (unaligned rows):
        // 32 columns at a time, accumulator handed back after the last TMEM
        // read.
#pragma unroll 1
        for (int cc = 0; cc < Cfg::kBN / 32; ++cc) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(t_row + cc * 32, r);
          tmem_wait_ld();
          if ((Cfg::kIssuers == 2 && cc == Cfg::kBN / 64 - 1) || cc == Cfg::kBN / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
              mbar_arrive_cluster_relaxed(cc == Cfg::kBN / 32 - 1 ? acc_empty_leader1
                                                                  : acc_empty_leader0);
          }
          const int col0 = n0 + tmem_block(cc / 2) * 64 + (cc % 2) * 32;
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
    if constexpr (kOut == 2) {
      if (p.rq_amax) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) rq_max = fmaxf(rq_max, __shfl_xor_sync(0xffffffffu, rq_max, o));
        // Non-negative floats order like their bit patterns.
        if (lane == 0 && rq_max > 0.0f) atomicMax(p.rq_amax, __float_as_uint(rq_max));
      }
    }
  }

  if (Cfg::kEpiBytes > 0 && ((warp >= 2 && warp <= 5) || warp >= 11) && (threadIdx.x % 32) == 0)
    tma_store_wait_all<0>();  // output stores done before shared memory is released
  tc_fence_before();
  cluster_sync();  // the leader's MMAs into both TMEMs are drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

template <int kFmt, int kOut>
static cudaError_t launch_pair_one(const GemmParams& p, int grid, cudaStream_t stream) {
  using Cfg = PairCfg<kFmt>;
  auto kern = gemm_pair_kernel<kFmt, kOut>;
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
  kern<<<grid, kOut >= 2 ? pair_threads<kOut>() : Cfg::kThreads, Cfg::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm_pair(const GemmParams& p, int fmt, int out_kind, int grid,
                             cudaStream_t stream) {
  if (fmt == kFmtNvfp4) {
    if (out_kind == 3) return launch_pair_one<kFmtNvfp4, 3>(p, grid, stream);
    if (out_kind == 2) return launch_pair_one<kFmtNvfp4, 2>(p, grid, stream);
    return out_kind == 1 ? launch_pair_one<kFmtNvfp4, 1>(p, grid, stream)
                         : launch_pair_one<kFmtNvfp4, 0>(p, grid, stream);
  }
  if (out_kind == 2) return cudaErrorInvalidValue;
  if (out_kind == 3)
    return fmt == kFmtMxfp4 ? launch_pair_one<kFmtMxfp4, 3>(p, grid, stream)
                            : launch_pair_one<kFmtMxfp8, 3>(p, grid, stream);
  if (fmt == kFmtMxfp4)
    return out_kind == 1 ? launch_pair_one<kFmtMxfp4, 1>(p, grid, stream)
                         : launch_pair_one<kFmtMxfp4, 0>(p, grid, stream);
  return out_kind == 1 ? launch_pair_one<kFmtMxfp8, 1>(p, grid, stream)
                       : launch_pair_one<kFmtMxfp8, 0>(p, grid, stream);
}

int pair_tile_m() { return 2 * PairCfg<kFmtNvfp4>::kBM; }
int pair_tile_n() { return PairCfg<kFmtNvfp4>::kBN; }
int pair_sf_chunks_per_stage(int fmt) {
  return fmt == kFmtNvfp4 ? PairCfg<kFmtNvfp4>::kSfChunks
                          : (fmt == kFmtMxfp4 ? PairCfg<kFmtMxfp4>::kSfChunks
                                              : PairCfg<kFmtMxfp8>::kSfChunks);
}

}  // namespace qg
