// gemm_skinny.cu -- decode-shaped NVFP4 GEMM (few activation rows, large
// weight matrix), HBM-bound.
//
// C[m, n] = (ts_x * ts_w) * sum_k x(m,k) w(n,k), m <= 128, computed as
// C^T = W . X^T so the weight rows fill the tensor core's M = 128 side and the
// activation rows its N side (16 / 32 / 64 / 128).  The reference has no
// kernel for this shape (its harness only runs square problems,
// GEMMquant_sm110/src/quant_gemm_bench.cu:3038-3079); BASELINE config 4 names
// it.  The weights are streamed once from HBM.  Work is (weight-tile,
// K-block) units: every CTA owns floor(T / G) whole tiles, and the units of
// the remaining T mod G tiles are spread evenly over all CTAs (stream-K), so
// the 224 x 16 units of N = 28672, K = 8192 split into one whole tile plus
// ~8 units per CTA on 148 SMs.  A tile that one CTA owns is scaled and
// written to C by that CTA; a tile split between CTAs is summed by the last
// of them to finish (see the epilogue), while the whole tiles stream.
// The activation quantisation runs in the same cooperative grid (see
// quantize_phase), so a call is one launch: no memset, quantiser, reduction
// or finishing kernel.
//
// Roles (10 warps): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2..9 first quantise the activations, then warps 2..5 are the
// epilogue (one TMEM quadrant each: lane = weight row) and warps 6..9 the
// scale stagers (tcgen05.st, as in gemm_solo.cu).  The accumulator is double
// buffered so a segment's reduction overlaps the next segment's mainloop.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qg_codec.cuh"
#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

#ifndef QG_SKINNY_L2_AHEAD
#define QG_SKINNY_L2_AHEAD 8
#endif

// Upper bound of the GEMM grid; sizes the partial-tile workspace.
constexpr int kSkinnyMaxCtas = 256;

template <int kN>
struct SkinnyCfg {
  static constexpr int kBM = 128;        // weight rows per tile
  static constexpr int kBoxBytes = 128;  // one SWIZZLE_128B box: 256 fp4 of K
  static constexpr int kBoxes = 2;       // boxes per stage: 512 of K
  static constexpr int kBKBytes = kBoxes * kBoxBytes;
  // A stage carries 8 MMAs: the serial per-stage cost of the issue loops
  // (barrier waits, commit) is paid once per 32 KB of weights.
  static constexpr int kMmaPerStage = 4 * kBoxes;
  static constexpr int kSfChunks = 4 * kBoxes;  // 512-byte chunks, 64 of K each
  static constexpr int kWBox = kBM * kBoxBytes;
  static constexpr int kXBox = kN * kBoxBytes;
  static constexpr int kWBytes = kWBox * kBoxes;
  static constexpr int kXBytes = kXBox * kBoxes;
  static constexpr int kSfwBytes = kSfChunks * 512;
  static constexpr int kSfxBytes = kSfChunks * 512;
  static constexpr int kStageTx = kWBytes + kXBytes + kSfwBytes + kSfxBytes;
  static constexpr int kStageBytes = (kStageTx + 1023) / 1024 * 1024;
  static constexpr int kSfStageCols = 8 * kSfChunks;  // 4 weight + 4 activation per chunk
  static constexpr int kTmemSfBase = 2 * kN < 64 ? 64 : 2 * kN;
  static constexpr int kTmemCols = 512;
  static constexpr int kSmemStages = (232448 - 512 - 1024) / kStageBytes;
  static constexpr int kTmemStages = (kTmemCols - kTmemSfBase) / kSfStageCols;
  static constexpr int kStages0 = kSmemStages < kTmemStages ? kSmemStages : kTmemStages;
  static constexpr int kStages = kStages0 < 8 ? kStages0 : 8;
  static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
  static_assert(kStages >= 2, "pipeline depth");
  static_assert(2 * kN <= kTmemSfBase, "accumulators");
  static_assert(kTmemSfBase + kStages * kSfStageCols <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr int kThreads = 320;
};

// Work of one CTA.  With T tiles over G CTAs, every CTA owns w = T / G
// whole tiles (the last T - (T mod G) tiles, contiguous per CTA) and an
// equal contiguous share of the units (tile, K block) of the first T mod G
// tiles, the "split region" (stream-K).  A split tile is shared by at most a
// few neighbouring CTAs and summed by the last of them to finish it.
struct UnitRange {
  int nkb;
  int split_tiles, split_units;  // the split region: tiles [0, split_tiles)
  int su0, su1;                  // this CTA's units of it
  int wt0, wn;                   // this CTA's whole tiles [wt0, wt0 + wn)
  __device__ __forceinline__ void init(int num_tiles, int num_kb, int c, int g) {
    nkb = num_kb;
    wn = num_tiles / g;
    split_tiles = num_tiles - wn * g;
    // Every CTA must own at least one split unit when there is a split
    // region (the contributor count of a split tile assumes it): with fewer
    // split units than CTAs, fall back to stream-K over all units (the host
    // launches at most num_tiles * num_kb CTAs).
    if (split_tiles > 0 && split_tiles * nkb < g) {
      wn = 0;
      split_tiles = num_tiles;
    }
    split_units = split_tiles * nkb;
    su0 = static_cast<int>(static_cast<int64_t>(split_units) * c / g);
    su1 = static_cast<int>(static_cast<int64_t>(split_units) * (c + 1) / g);
    wt0 = split_tiles + c * wn;
  }
  __device__ __forceinline__ int units() const { return su1 - su0 + wn * nkb; }
  // CTA owning split-region unit u, and the first split tile of CTA c.
  __device__ __forceinline__ int contributor(int64_t u, int g) const {
    return static_cast<int>(((u + 1) * g - 1) / split_units);
  }
  __device__ __forceinline__ int first_split_tile(int c, int g) const {
    return static_cast<int>(static_cast<int64_t>(split_units) * c / g / nkb);
  }
};

// Order in which a CTA walks its work: the split segments first -- the one
// of its LAST split tile, then the one of its first, then any split tiles
// between (whole within the range) -- and the whole tiles last.  The split
// tiles' fixups (the last contributor sums the partial slices) therefore
// overlap the streaming of the whole tiles instead of trailing the kernel,
// whose last segments are stored straight to C.
struct SegCursor {
  int nkb, su0, su1, wt0, wn;
  int tile_lo, tile_hi, nsplit;
  int i, t, kb, kb_end;  // segment index, its tile, current / end K block
  __device__ __forceinline__ void init(const UnitRange& r) {
    nkb = r.nkb;
    su0 = r.su0;
    su1 = r.su1;
    wt0 = r.wt0;
    wn = r.wn;
    if (su1 > su0) {
      tile_lo = su0 / nkb;
      tile_hi = (su1 - 1) / nkb;
      nsplit = tile_hi - tile_lo + 1;
    } else {
      tile_lo = tile_hi = -1;
      nsplit = 0;
    }
    i = 0;
    if (nseg() > 0) enter();
  }
  __device__ __forceinline__ int nseg() const { return nsplit + wn; }
  __device__ __forceinline__ bool split(int s) const { return s < nsplit; }
  __device__ __forceinline__ int tile_of(int s) const {
    if (s >= nsplit) return wt0 + (s - nsplit);
    if (tile_hi == tile_lo) return tile_lo;
    return s == 0 ? tile_hi : (s == 1 ? tile_lo : tile_lo + s - 1);
  }
  __device__ __forceinline__ int kb_lo(int s) const {
    const int tt = tile_of(s);
    return (s < nsplit && tt == tile_lo) ? su0 - tt * nkb : 0;
  }
  __device__ __forceinline__ int kb_hi(int s) const {
    const int tt = tile_of(s);
    return (s < nsplit && tt == tile_hi) ? su1 - tt * nkb : nkb;
  }
  __device__ __forceinline__ void enter() {
    t = tile_of(i);
    kb = kb_lo(i);
    kb_end = kb_hi(i);
  }
  // Step to the next unit; false past the end of the work.
  __device__ __forceinline__ bool next() {
    if (++kb < kb_end) return true;
    if (++i >= nseg()) return false;
    enter();
    return true;
  }
};

// Diagnostic stamp (kDiag bit 6): CTA (kDiag >> 16) writes %globaltimer into
// slot `i` of the last (never used by a launched CTA) partial slice pair.
__device__ __forceinline__ void trace_cta(const SkinnyParams& p, int i) {
  if (kDiag & 64u)
    reinterpret_cast<unsigned long long*>(p.part + static_cast<int64_t>(kSkinnyMaxCtas - 1) * 2 * p.m * 128)[i] = globaltimer_ns();
}
__device__ __forceinline__ void trace(const SkinnyParams& p, int i) {
  if ((kDiag & 64u) && blockIdx.x == (kDiag >> 16) && i < 512)
    reinterpret_cast<unsigned long long*>(p.part + static_cast<int64_t>(kSkinnyMaxCtas - 1) * 2 * p.m * 128)[i] = globaltimer_ns();
}

// ------------------------------------------------------------------ activation quantiser
// Run by the 256 threads of warps 2..9 of every CTA before their GEMM roles,
// while warp 0 already streams the first weight stages.  make_nvfp4_reference
// (GEMMsm110/include/requant/nvfp4_reference.cuh:76-112) bit for bit, MMA
// layout:
//   1. each CTA reduces the amax of its contiguous range of 16-element
//      blocks into amax_part[cta]; grid arrival #1;
//   2. every CTA reduces amax_part, quantises its range into xq / xsf,
//      zeroes its share of the padding scale slots and of the tile counters;
//      grid arrival #2, after which x_ready lets the producer issue the
//      activation loads.
// The last CTA to leave resets the arrival counters for the next call.
// Returns false when a grid arrival timed out (status recorded).
constexpr int kQuantThreads = 256;
constexpr uint32_t kQuantBar = 1;  // named barrier id of warps 2..9

template <bool kBf16>
__device__ bool quantize_phase(const SkinnyParams& p, int qt, float* red,
                               volatile uint32_t* abort_flag, uint64_t* x_loaded,
                               uint64_t* x_ready) {
  constexpr int kFly = kBf16 ? 4 : 2;  // blocks in flight per thread
  const int G = gridDim.x, c = blockIdx.x;
  const int64_t sfk = p.k / 16;
  const int64_t nblocks = static_cast<int64_t>(p.m) * sfk;
  const int64_t b0 = nblocks * c / G, b1 = nblocks * (c + 1) / G;

  // The first kFly blocks of a thread stay in registers for the second pass
  // (decode-sized x: usually all of them), later ones are read again.
  float mx = 0.0f;
  RawBlock<kBf16> keep[kFly];
  const int64_t chunk = static_cast<int64_t>(kFly) * kQuantThreads;
#pragma unroll
  for (int f = 0; f < kFly; ++f)
    if (b0 + qt + f * kQuantThreads < b1) keep[f].load(p.x, b0 + qt + f * kQuantThreads);
#pragma unroll
  for (int f = 0; f < kFly; ++f) {
    if (b0 + qt + f * kQuantThreads >= b1) break;
    float v[16];
    keep[f].decode(v);
#pragma unroll
    for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
  }
  for (int64_t base = b0 + qt + chunk; base < b1; base += chunk) {
    RawBlock<kBf16> r[kFly];
#pragma unroll
    for (int f = 0; f < kFly; ++f)
      if (base + f * kQuantThreads < b1) r[f].load(p.x, base + f * kQuantThreads);
#pragma unroll
    for (int f = 0; f < kFly; ++f) {
      if (base + f * kQuantThreads >= b1) break;
      float v[16];
      r[f].decode(v);
#pragma unroll
      for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((qt & 31) == 0) red[qt >> 5] = mx;
  named_bar_sync(kQuantBar, kQuantThreads);
  if (qt == 0) {
    trace(p, 4);
    mbar_arrive(x_loaded);
    float a = 0.0f;
    for (int w = 0; w < kQuantThreads / 32; ++w) a = fmaxf(a, red[w]);
    p.amax_part[c] = a;
    const bool ok = grid_arrive_wait(&p.sync[0], G, p.timeout_ns, abort_flag, p.status,
                                     kDevTimeoutGridSync);
    red[8] = ok ? 1.0f : 0.0f;
    trace(p, 5);
  }
  named_bar_sync(kQuantBar, kQuantThreads);
  if (red[8] == 0.0f) return false;
  if (qt < 32) {
    float a = 0.0f;
    for (int r = qt; r < G; r += 32) a = fmaxf(a, __ldcg(p.amax_part + r));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (qt == 0) red[9] = a;
  }
  named_bar_sync(kQuantBar, kQuantThreads);
  const float amax = red[9];
  const float ts = amax > 0.0f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  const float inv_ts = __fdiv_rn(1.0f, ts);
  if (c == 0 && qt == 0) *p.x_ts = ts;

  const int64_t sf_blocks = (sfk + 3) / 4;  // one 128-row block: m <= 128
  auto encode = [&](const RawBlock<kBf16>& r, int64_t b) {
    float v[16];
    r.decode(v);
    uint32_t lo, hi;
    const uint32_t sbits = nvfp4_encode_block(v, inv_ts, lo, hi);
    reinterpret_cast<uint2*>(p.xq)[b] = make_uint2(lo, hi);
    const int64_t row = b / sfk, sc = b - row * sfk;
    p.xsf[mma_scale_offset(row, sc, 1, sf_blocks, 1)] = static_cast<uint8_t>(sbits);
  };
#pragma unroll
  for (int f = 0; f < kFly; ++f)
    if (b0 + qt + f * kQuantThreads < b1) encode(keep[f], b0 + qt + f * kQuantThreads);
  for (int64_t base = b0 + qt + chunk; base < b1; base += chunk) {
    RawBlock<kBf16> r[kFly];
#pragma unroll
    for (int f = 0; f < kFly; ++f)
      if (base + f * kQuantThreads < b1) r[f].load(p.x, base + f * kQuantThreads);
#pragma unroll
    for (int f = 0; f < kFly; ++f)
      if (base + f * kQuantThreads < b1) encode(r[f], base + f * kQuantThreads);
  }
  if (qt == 0) trace(p, 6);
  // Padding scale slots (rows >= m, scale columns >= k/16) read as zero.
  const int64_t cols_pad = sf_blocks * 4, npad = 128 * cols_pad;
  const int64_t gt = static_cast<int64_t>(c) * kQuantThreads + qt, gstride = static_cast<int64_t>(G) * kQuantThreads;
  if (npad != nblocks) {
    for (int64_t i = gt; i < npad; i += gstride) {
      const int64_t row = i / cols_pad, sc = i - row * cols_pad;
      if (row >= p.m || sc >= sfk) p.xsf[mma_scale_offset(row, sc, 1, sf_blocks, 1)] = 0u;
    }
  }
  for (int64_t i = gt; i < static_cast<int64_t>(p.num_tiles) * 4; i += gstride) p.cnt[i] = 0u;
  asm volatile("fence.proxy.async.global;" ::: "memory");  // xq / xsf are read by TMA
  named_bar_sync(kQuantBar, kQuantThreads);
  if (qt == 0) trace(p, 7);
  if (qt == 0) {
    const bool ok = grid_arrive_wait(&p.sync[1], G, p.timeout_ns, abort_flag, p.status,
                                     kDevTimeoutGridSync);
    red[8] = ok ? 1.0f : 0.0f;
    trace(p, 8);
    if (ok) {
      mbar_arrive(x_ready);
      if (atomicAdd(&p.sync[2], 1u) == static_cast<uint32_t>(G - 1)) {
        p.sync[0] = 0u;
        p.sync[1] = 0u;
        p.sync[2] = 0u;
      }
    }
  }
  named_bar_sync(kQuantBar, kQuantThreads);
  return red[8] != 0.0f;
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
  uint64_t* x_ready = acc_full + 5;   // quantised activations visible grid-wide
  uint64_t* x_loaded = acc_full + 6;  // this CTA's quantiser has read its activations
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 7);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* qred = reinterpret_cast<float*>(tmem_slot + 2);  // [10] quantiser scratch

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
    mbar_init(x_ready, 1);
    mbar_init(x_loaded, 1);
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
  if (threadIdx.x == 0) trace_cta(p, 768 + blockIdx.x);
  UnitRange ur;
  ur.init(p.num_tiles, p.num_k_blocks, static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x));

  bool quant_ok = true;
  if (warp >= 2) {
    const int qt = threadIdx.x - 64;
    if (kDiag & 4096u) {
      // Diagnostic: the activations taken as already quantised (results
      // wrong by design), to weigh the in-kernel quantisation's cost.
      if (qt == 0) {
        mbar_arrive(x_loaded);
        mbar_arrive(x_ready);
      }
    } else {
      quant_ok = p.x_bf16 ? quantize_phase<true>(p, qt, qred, abort_flag, x_loaded, x_ready)
                          : quantize_phase<false>(p, qt, qred, abort_flag, x_loaded, x_ready);
    }
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();  // weights: streamed once
      const uint64_t pol_x = l2_policy_evict_last();   // activations: reused by all CTAs
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      // The first kStages stages get their weight loads at once and the
      // next kL2Ahead units' weights are prefetched into L2; the activation
      // loads wait for the in-kernel quantiser (x_ready), so the weight
      // stream runs while the activations are being quantised.  On a
      // quantiser timeout the deferred loads are still issued (the buffers
      // are valid memory) so every armed stage completes before exit.
      constexpr int kL2Ahead = QG_SKINNY_L2_AHEAD;  // units (32 KB of weights each)
      int deferred = 0;
      int dkb[Cfg::kStages];
      auto issue_x = [&](int s, int k_blk) {
        uint8_t* sx = smem + s * Cfg::kStageBytes + Cfg::kWBytes;
        uint8_t* ssfx = sx + Cfg::kXBytes + Cfg::kSfwBytes;
        tma_load_3d(ssfx, &p.tm_sfx, &full_bar[s], 0, 0, k_blk * Cfg::kSfChunks, pol_x);
#pragma unroll
        for (int h = 0; h < Cfg::kBoxes; ++h)
          tma_load_2d(sx + h * Cfg::kXBox, &p.tm_x, &full_bar[s],
                      k_blk * Cfg::kBKBytes + h * Cfg::kBoxBytes, 0, pol_x);
      };
      bool dep_done = false;
      auto release_deferred = [&](SegCursor ahead, bool more) {
        for (int i = 0; more && i < kL2Ahead; ++i) {
          tma_prefetch_l2_3d(&p.tm_sfw, 0, ahead.t, ahead.kb * Cfg::kSfChunks);
#pragma unroll
          for (int h = 0; h < Cfg::kBoxes; ++h)
            tma_prefetch_l2_2d(&p.tm_w, ahead.kb * Cfg::kBKBytes + h * Cfg::kBoxBytes,
                               ahead.t * Cfg::kBM);
          more = ahead.next();
        }
        if (!mbar_wait_bounded(x_ready, 0, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutProducer))
          ok = false;
        asm volatile("fence.proxy.async.global;" ::: "memory");
        trace(p, 2);
        for (int s = 0; s < deferred; ++s) issue_x(s, dkb[s]);
        dep_done = true;
      };
      // The weight stream starts once this CTA's quantiser has read its
      // share of the activations, so those reads do not queue behind it.
      if (!mbar_wait_bounded(x_loaded, 0, p.timeout_ns, abort_flag, p.status,
                             kDevTimeoutProducer))
        ok = false;
      SegCursor cur;
      cur.init(ur);
      bool more = ok && cur.nseg() > 0;
      for (int g = 0; more; ++g) {
        if (!dep_done && g == Cfg::kStages) {
          release_deferred(cur, true);
          if (!ok) break;
        }
        if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* sw = smem + stage * Cfg::kStageBytes;
        uint8_t* ssfw = sw + Cfg::kWBytes + Cfg::kXBytes;
        trace(p, 16 + g);
        mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageTx);
        tma_load_3d(ssfw, &p.tm_sfw, &full_bar[stage], 0, cur.t, cur.kb * Cfg::kSfChunks, pol_w);
#pragma unroll
        for (int h = 0; h < Cfg::kBoxes; ++h)
          tma_load_2d(sw + h * Cfg::kWBox, &p.tm_w, &full_bar[stage],
                      cur.kb * Cfg::kBKBytes + h * Cfg::kBoxBytes, cur.t * Cfg::kBM, pol_w);
        if (dep_done) {
          issue_x(stage, cur.kb);
        } else {
          dkb[deferred++] = cur.kb;
        }
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        more = cur.next();
        if (++stage == Cfg::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!dep_done) release_deferred(cur, false);
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
      // The issue loop is the kernel's serial path (one thread, a dependent
      // instruction chain): segments are walked outside, the per-unit body
      // is a wait, eight MMAs and a commit, with descriptors and scale
      // columns stepped by constants.
      const uint32_t idesc = make_idesc_block_scaled(Cfg::kBM, kN, 1u, 0u, 0u, 0u);
      const bool skip_mma = (kDiag & 2u) != 0;
      const uint64_t wdesc0 = make_smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      const uint64_t xdesc0 = make_smem_desc(smem_u32(smem + Cfg::kWBytes), 16, 1024, kSwizzle128B);
      constexpr uint64_t kStageDesc = Cfg::kStageBytes >> 4;
      bool ok = true;
      int stage = 0, g = 0;
      uint32_t phase = 0;
      uint64_t wdesc = wdesc0, xdesc = xdesc0;
      uint32_t sfw_col = tmem_base + Cfg::kTmemSfBase;
      SegCursor order;
      order.init(ur);
      for (int seg = 0; ok && seg < order.nseg(); ++seg) {
        const int t = order.tile_of(seg);
        const int kb_lo = order.kb_lo(seg);
        const int kb_hi = order.kb_hi(seg);
        const int buf = seg & 1;
        if (!mbar_wait_bounded(&acc_empty[buf], ((seg >> 1) & 1) ^ 1u, p.timeout_ns, abort_flag,
                               p.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * kN);
        uint32_t acc = 0;
        for (int j = kb_lo; j < kb_hi; ++j, ++g) {
          // sf_ready is arrived by the stagers only after they observed
          // full_bar, so it also orders the TMA data of the stage.
          if (!mbar_wait_bounded(&sf_ready[stage], phase, p.timeout_ns, abort_flag, p.status,
                                 kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int i = 0; i < Cfg::kMmaPerStage; ++i) {
            if (skip_mma) break;
            // MMA i: box i / 4, 32-byte K step (i % 4) inside the 128-byte row.
            const uint64_t wo = static_cast<uint64_t>((i / 4) * (Cfg::kWBox >> 4) + (i % 4) * 2);
            const uint64_t xo = static_cast<uint64_t>((i / 4) * (Cfg::kXBox >> 4) + (i % 4) * 2);
            mma_mxf4nvf4(d_tmem, wdesc + wo, xdesc + xo, idesc, sfw_col + i * 4,
                         sfw_col + 4 * Cfg::kSfChunks + i * 4, acc);
            acc = 1;
          }
          tc_commit(&empty_bar[stage]);
          trace(p, 320 + g);
          if (++stage == Cfg::kStages) {
            stage = 0;
            phase ^= 1u;
            wdesc = wdesc0;
            xdesc = xdesc0;
            sfw_col = tmem_base + Cfg::kTmemSfBase;
          } else {
            wdesc += kStageDesc;
            xdesc += kStageDesc;
            sfw_col += Cfg::kSfStageCols;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
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
    const int my_units = ur.units();
    for (int u = 0; quant_ok && u < my_units; ++u) {
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(&full_bar[stage], phase);
      const uint8_t* ssfw = smem + stage * Cfg::kStageBytes + Cfg::kWBytes + Cfg::kXBytes;
      const uint8_t* ssfx = ssfw + Cfg::kSfwBytes;
      // Weight scales in columns [0, 32), activation scales in [32, 64) of
      // the stage's slot, written with ONE tcgen05.st (a store costs about
      // the same whatever its width).
      uint32_t v[8 * Cfg::kSfChunks];
      uint32_t* a = v;
      uint32_t* b = v + 4 * Cfg::kSfChunks;
#pragma unroll
      for (int c = 0; c < Cfg::kSfChunks; ++c) {
        const uint4 x = lds128(ssfw + c * 512 + lane * 16);
        const uint4 w = lds128(ssfx + c * 512 + lane * 16);
        a[4 * c] = x.x; a[4 * c + 1] = x.y; a[4 * c + 2] = x.z; a[4 * c + 3] = x.w;
        b[4 * c] = w.x; b[4 * c + 1] = w.y; b[4 * c + 2] = w.z; b[4 * c + 3] = w.w;
      }
      const uint32_t col = Cfg::kTmemSfBase + stage * Cfg::kSfStageCols;
      if (!(kDiag & 1u)) {
        tmem_st_32x32b<8 * Cfg::kSfChunks>(t_quad + col, v);
        tmem_wait_st();
      }
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
    if (quad == 0 && lane == 0) trace(p, 3);
    const float alpha = __ldcg(p.x_ts) * (p.w_ts ? *p.w_ts : 1.0f);
    const int grid = static_cast<int>(gridDim.x);
    auto first_tile = [&](int c) { return ur.first_split_tile(c, grid); };
    auto store_c = [&](int m, int n, float v) {
      if (p.out_bf16)
        reinterpret_cast<__nv_bfloat16*>(p.c)[static_cast<int64_t>(m) * p.ldc + n] =
            __float2bfloat16_rn(v);
      else
        reinterpret_cast<float*>(p.c)[static_cast<int64_t>(m) * p.ldc + n] = v;
    };
    SegCursor order;
    order.init(ur);
    const int my_first = order.tile_lo;
    for (int seg = 0; quant_ok && seg < order.nseg(); ++seg) {
      const int t = order.tile_of(seg);
      const int buf = seg & 1;
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded<false, 128>(&acc_full[buf], (seg >> 1) & 1, p.timeout_ns,
                                           abort_flag, p.status, kDevTimeoutEpilogue);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(&acc_full[buf], (seg >> 1) & 1);
      tc_fence_after();
      if (quad == 0 && lane == 0) trace(p, 120 + seg);
      const int col = quad * 32 + lane;
      const int n = t * Cfg::kBM + col;
      const bool n_ok = n < p.n;
      // Contributors of a split tile (whole tiles: this CTA alone).
      const bool split = order.split(seg);
      const int cf = split ? ur.contributor(static_cast<int64_t>(t) * ur.nkb, grid)
                           : static_cast<int>(blockIdx.x);
      const int cl = split ? ur.contributor(static_cast<int64_t>(t + 1) * ur.nkb - 1, grid)
                           : static_cast<int>(blockIdx.x);
      float* mine = p.part + static_cast<int64_t>(blockIdx.x * 2 + (t == my_first ? 0 : 1)) *
                                 p.m * Cfg::kBM;
      // TMEM reads queue behind the MMAs already issued for the next
      // segment, so each wait can cost the queued MMA time: read up to 64
      // columns per wait (one wait for kN <= 64, two for kN = 128).
      constexpr int kGroup = kN < 64 ? kN : 64;
      // One destination per segment: C (scaled, row stride ldc) for a whole
      // tile, else this CTA's fp32 partial slice (row stride 128).  The
      // per-element code is kept to a multiply, an address step and a store:
      // the unrolled epilogue competes for instruction cache with four other
      // roles, and a fetch miss under the weight stream costs microseconds.
      const bool whole = cf == cl;
      const bool st_ok = !(kDiag & 8u) && (!whole || n_ok);
      const float scale = whole ? alpha : 1.0f;
      const bool bf16_dst = whole && p.out_bf16;
      const int64_t stride = whole ? p.ldc : Cfg::kBM;
      float* dstf = whole ? reinterpret_cast<float*>(p.c) + n : mine + col;
      __nv_bfloat16* dstb = reinterpret_cast<__nv_bfloat16*>(p.c) + n;
      const int mrows = p.m;
      const int n_tail = t * Cfg::kBM + quad * 32;
      const bool bf16_tail = bf16_dst && seg == order.nseg() - 1 && p.vec_ok && n_tail + 32 <= p.n;
#pragma unroll
      for (int gc = 0; gc < kN / kGroup; ++gc) {
        uint32_t r[kGroup];
#pragma unroll
        for (int cc = 0; cc < kGroup / 16; ++cc)
          tmem_ld_32x32b_x16(t_quad + static_cast<uint32_t>(buf * kN + gc * kGroup + cc * 16),
                             *reinterpret_cast<uint32_t(*)[16]>(r + cc * 16));
        tmem_wait_ld();
        if (gc == kN / kGroup - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        if (gc == 0 && quad == 0 && lane == 0) trace(p, 110 + seg);
        if (!st_ok) continue;
        if (bf16_tail) {
          // Final segment (a whole tile): the stage ring is idle (every load
          // has been consumed by the MMAs this wait covered), so this warp
          // transposes its 32 columns x kGroup rows through it and writes C
          // in 16-byte row pieces: 8 lanes' worth of stores per row instead
          // of one 2-byte store per lane and row.
          uint8_t* tbuf = smem + quad * (kGroup * 64);
          __syncwarp();
#pragma unroll
          for (int j = 0; j < kGroup; ++j)
            *reinterpret_cast<__nv_bfloat16*>(tbuf + j * 64 + lane * 2) =
                __float2bfloat16_rn(__uint_as_float(r[j]) * scale);
          __syncwarp();
          const int c16 = (lane & 3) * 16;
          uint8_t* crow = reinterpret_cast<uint8_t*>(p.c) + static_cast<int64_t>(n_tail) * 2 + c16;
#pragma unroll
          for (int it = 0; it < kGroup / 8; ++it) {
            const int row = it * 8 + (lane >> 2);
            const int mm = gc * kGroup + row;
            const uint4 v = *reinterpret_cast<const uint4*>(tbuf + row * 64 + c16);
            if (mm < mrows) *reinterpret_cast<uint4*>(crow + static_cast<int64_t>(mm) * p.ldc * 2) = v;
          }
          continue;
        }
        if (bf16_dst) {
#pragma unroll
          for (int j = 0; j < kGroup; ++j)
            if (gc * kGroup + j < mrows)
              dstb[(gc * kGroup + j) * stride] = __float2bfloat16_rn(__uint_as_float(r[j]) * scale);
        } else if (whole) {
#pragma unroll
          for (int j = 0; j < kGroup; ++j)
            if (gc * kGroup + j < mrows) dstf[(gc * kGroup + j) * stride] = __uint_as_float(r[j]) * scale;
        } else {
#pragma unroll
          for (int j = 0; j < kGroup; ++j)
            if (gc * kGroup + j < mrows) __stcg(dstf + (gc * kGroup + j) * stride, __uint_as_float(r[j]));
        }
      }
      if (quad == 0 && lane == 0) trace(p, 100 + seg);
      if (cf == cl) continue;
      // Publish the slice and count this contributor with one acquire-release
      // atomic from lane 0: the warp barrier before it orders every lane's
      // slice stores ahead of the release (fence cumulativity), the one after
      // it orders every lane's slice reads behind the acquire.  Two full
      // fences here each cost ~2 us while the weight stream loads the memory
      // system.
      if (quad == 0 && lane == 0) trace(p, 300 + 4 * seg);
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atom_add_acq_rel_gpu(&p.cnt[t * 4 + quad], 1u);
      old = __shfl_sync(0xffffffffu, old, 0);
      __syncwarp();
      if (quad == 0 && lane == 0) trace(p, 301 + 4 * seg);
      if (old != static_cast<uint32_t>(cl - cf)) continue;
      if (quad == 0 && lane == 0) trace(p, 302 + 4 * seg);
      // Sum pass: a lane takes 8 adjacent columns of one row, a warp
      // instruction 8 rows x 32 columns; 4 steps x 3 contributors x 32 bytes
      // are in flight per lane before the adds (in contributor order), and
      // each step ends in one 16-byte (bf16) or two (fp32) stores per lane.
      {
        const int sub = lane >> 2, c8 = (lane & 3) * 8;
        const int64_t slice = static_cast<int64_t>(p.m) * Cfg::kBM;
        const int nb = t * Cfg::kBM + quad * 32 + c8;
        const bool vec = p.vec_ok && nb + 8 <= p.n;
#pragma unroll 1
        for (int m0 = 0; m0 < p.m; m0 += 32) {
          float acc[4][8];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[i][e] = 0.0f;
#pragma unroll 1
          for (int c = cf; c <= cl; c += 3) {
            // Up to three contributors' loads in flight at once (a split
            // tile has two or three): one memory round per 32 rows.
            const bool two = c + 1 <= cl, three = c + 2 <= cl;
            const float* s0 = p.part + (c * 2 + (t == first_tile(c) ? 0 : 1)) * slice + quad * 32 + c8;
            const float* s1 = two ? p.part + ((c + 1) * 2 + (t == first_tile(c + 1) ? 0 : 1)) * slice +
                                        quad * 32 + c8
                                  : s0;
            const float* s2 = three ? p.part + ((c + 2) * 2 + (t == first_tile(c + 2) ? 0 : 1)) * slice +
                                          quad * 32 + c8
                                    : s0;
            float4 v0[4][2], v1[4][2], v2[4][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int m = m0 + i * 8 + sub;
              const bool ok = m < p.m;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                v0[i][h] = ok ? __ldcg(reinterpret_cast<const float4*>(s0 + m * Cfg::kBM) + h)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
                v1[i][h] = ok && two ? __ldcg(reinterpret_cast<const float4*>(s1 + m * Cfg::kBM) + h)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                v2[i][h] = ok && three ? __ldcg(reinterpret_cast<const float4*>(s2 + m * Cfg::kBM) + h)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                acc[i][4 * h] += v0[i][h].x; acc[i][4 * h + 1] += v0[i][h].y;
                acc[i][4 * h + 2] += v0[i][h].z; acc[i][4 * h + 3] += v0[i][h].w;
                if (two) {
                  acc[i][4 * h] += v1[i][h].x; acc[i][4 * h + 1] += v1[i][h].y;
                  acc[i][4 * h + 2] += v1[i][h].z; acc[i][4 * h + 3] += v1[i][h].w;
                }
                if (three) {
                  acc[i][4 * h] += v2[i][h].x; acc[i][4 * h + 1] += v2[i][h].y;
                  acc[i][4 * h + 2] += v2[i][h].z; acc[i][4 * h + 3] += v2[i][h].w;
                }
              }
          }
          if (quad == 0 && lane == 0 && m0 == 0) trace(p, 303 + 4 * seg);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = m0 + i * 8 + sub;
            if (m >= p.m) continue;
            if (vec) {
              if (p.out_bf16) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const __nv_bfloat162 h2 =
                      __floats2bfloat162_rn(acc[i][2 * e] * alpha, acc[i][2 * e + 1] * alpha);
                  w[e] = *reinterpret_cast<const uint32_t*>(&h2);
                }
                *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.c) +
                                          static_cast<int64_t>(m) * p.ldc + nb) =
                    make_uint4(w[0], w[1], w[2], w[3]);
              } else {
                float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.c) +
                                                        static_cast<int64_t>(m) * p.ldc + nb);
                dst[0] = make_float4(acc[i][0] * alpha, acc[i][1] * alpha, acc[i][2] * alpha,
                                     acc[i][3] * alpha);
                dst[1] = make_float4(acc[i][4] * alpha, acc[i][5] * alpha, acc[i][6] * alpha,
                                     acc[i][7] * alpha);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                if (nb + e < p.n) store_c(m, nb + e, acc[i][e] * alpha);
            }
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
  if (threadIdx.x == 0) trace_cta(p, 512 + blockIdx.x);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

template <int kN>
static cudaError_t launch_skinny_n(const SkinnyParams& p, int grid, cudaStream_t stream) {
  using Cfg = SkinnyCfg<kN>;
  auto kern = gemm_skinny_kernel<kN>;
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
  // Cooperative: every CTA is resident at once (the quantiser's grid-wide
  // arrivals rely on it), or the launch fails.
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
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
