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

#ifndef QG_SKINNY_WIDE
#define QG_SKINNY_WIDE 1
#endif
// Smallest MMA N (activation rows, padded) that takes the wide tiles.  A/B on
// one box, GB/s (m = 16 / 64 / 128): wide from N = 128: 5282 / 4132 / 4082;
// from N = 64: 5239 / 4444 / 4067; from N = 16: 4632 / 4434 / 4104 (at
// m = 16 the 128-row tiles' double-buffered accumulator and rolling L2 lead
// outweigh the activation bytes saved).
#ifndef QG_SKINNY_WIDE_MIN_N
#define QG_SKINNY_WIDE_MIN_N 64
#endif
// Register budgets that let one quantiser CTA (128 threads, <= 56
// registers) sit on an SM beside a GEMM CTA (320 threads, <= 152): an SM
// sub-partition holds three GEMM warps (3 x 152 x 32 registers) and one
// quantiser warp (56 x 32) in its 16384 registers, so the GEMM's CTAs start
// streaming weights at once on every SM instead of waiting for the
// quantiser CTAs there to exit.
#ifndef QG_SQ_MAXREG
#define QG_SQ_MAXREG 56
#endif
#ifndef QG_SKINNY_BOUNDS
#define QG_SKINNY_BOUNDS __maxnreg__(152)
#endif
#ifndef QG_SQ_THREADS
#define QG_SQ_THREADS 128
#endif
#ifndef QG_SKINNY_L2_ROLL
#define QG_SKINNY_L2_ROLL 1
#endif
#ifndef QG_SKINNY_L2_AHEAD
#define QG_SKINNY_L2_AHEAD 1
#endif
#ifndef QG_SKINNY_L2_ROLL_WIDE
#define QG_SKINNY_L2_ROLL_WIDE 0
#endif
#ifndef QG_SKINNY_L2_AHEAD_WIDE
#define QG_SKINNY_L2_AHEAD_WIDE 8
#endif

// Upper bound of the GEMM grid; sizes the partial-tile workspace.
constexpr int kSkinnyMaxCtas = 256;

// Tile shape by MMA N.  N <= 32: a tile is 128 weight rows, a stage 512 of
// K, two accumulator buffers (the next segment's MMAs overlap the epilogue).
// N = 64 and 128 ("wide"): a tile is 256 weight rows as two 128-row MMA halves
// that share the stage's activations, a stage 256 of K, one accumulator
// buffer of both halves.  The activation bytes per weight byte halve (16 KB
// per 32 KB of weights instead of 32 KB), so four stages fit in shared
// memory instead of three and more weight bytes are in flight per SM.
template <int kN>
struct SkinnyCfg {
  static constexpr int kH = (QG_SKINNY_WIDE && kN >= QG_SKINNY_WIDE_MIN_N) ? 2 : 1;  // 128-row halves per tile
  static constexpr int kBM = 128;        // weight rows per MMA (half)
  static constexpr int kTileRows = kBM * kH;
  static constexpr int kBoxBytes = 128;  // one SWIZZLE_128B box: 256 fp4 of K
  static constexpr int kBoxes = kH == 1 ? 2 : 1;  // boxes per stage: 512 / 256 of K
  static constexpr int kBKBytes = kBoxes * kBoxBytes;
  // A stage carries 8 MMAs: the serial per-stage cost of the issue loops
  // (barrier waits, commit) is paid once per 32 KB of weights.
  static constexpr int kSfChunks = 4 * kBoxes;  // 512-byte chunks, 64 of K each
  static constexpr int kMmaPerStage = kSfChunks * kH;
  static constexpr int kWBox = kBM * kBoxBytes;
  static constexpr int kXBox = kN * kBoxBytes;
  static constexpr int kWBytes = kWBox * kBoxes * kH;  // [box][half] boxes
  static constexpr int kXBytes = kXBox * kBoxes;
  static constexpr int kSfwBytes = kSfChunks * 512 * kH;  // [half][chunk]
  static constexpr int kSfxBytes = kSfChunks * 512;
  static constexpr int kStageTx = kWBytes + kXBytes + kSfwBytes + kSfxBytes;
  static constexpr int kStageBytes = (kStageTx + 1023) / 1024 * 1024;
  // A stage's scale slot: weight scales of each half, then the activation
  // scales (4 columns per chunk each), padded to a tcgen05.st width.
  static constexpr int kSfWords = 4 * kSfChunks * (kH + 1);
  static constexpr int kSfStageCols = kSfWords <= 32 ? 32 : kSfWords <= 64 ? 64 : 128;
  static constexpr int kAccBufs = kH == 1 ? 2 : 1;
  static constexpr int kAccCols = kAccBufs * kH * kN;
  static constexpr int kTmemSfBase = kAccCols < 64 ? 64 : kAccCols;
  static constexpr int kTmemCols = 512;
  static constexpr int kSmemStages = (232448 - 512 - 1024) / kStageBytes;
  static constexpr int kTmemStages = (kTmemCols - kTmemSfBase) / kSfStageCols;
  static constexpr int kStages0 = kSmemStages < kTmemStages ? kSmemStages : kTmemStages;
  static constexpr int kStages = kStages0 < 8 ? kStages0 : 8;
  static constexpr int kSmemBytes = kStages * kStageBytes + 512 + 1024;
  static_assert(kStages >= 2, "pipeline depth");
  static_assert(kAccCols <= kTmemSfBase, "accumulators");
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
    reinterpret_cast<unsigned long long*>(p.part + static_cast<int64_t>(kSkinnyMaxCtas - 1) * p.slices * p.m * 128)[i] = globaltimer_ns();
}
__device__ __forceinline__ void trace(const SkinnyParams& p, int i) {
  if ((kDiag & 64u) && blockIdx.x == (kDiag >> 16) && i < 512)
    reinterpret_cast<unsigned long long*>(p.part + static_cast<int64_t>(kSkinnyMaxCtas - 1) * p.slices * p.m * 128)[i] = globaltimer_ns();
}

// ------------------------------------------------------------------ activation quantiser
// Two small kernels run ahead of the GEMM in the stream, chained with
// programmatic dependent launch: make_nvfp4_reference
// (GEMMsm110/include/requant/nvfp4_reference.cuh:76-112) bit for bit, MMA
// layout.
//   1. skinny_amax_kernel: every CTA reduces the amax of its contiguous range
//      of 16-element blocks into amax_part[cta];
//   2. skinny_quant_kernel (launched while 1 runs, waits for it): every CTA
//      reduces amax_part, quantises its range into xq / xsf, zeroes its share
//      of the padding scale slots and of the tile counters; CTA 0 writes the
//      tensor scale.
// Both let their dependent start at once, so the GEMM's CTAs are resident
// and streaming weights while the activations are quantised; the GEMM waits
// for them (griddepcontrol.wait) only before its activation loads and its
// epilogue.  Measured against quantising inside the GEMM (two grid-wide
// arrivals under the weight stream): the GEMM without any quantisation is
// 17 % (m = 16) and 22 % (m = 128) faster, the bound this design aims at.
// The quantiser CTAs fit beside the GEMM's (register budgets above); their
// per-block work is kept short (hardware e2m1 conversion, a per-CTA table
// of the 127 possible element multipliers instead of a division per block).
constexpr int kSqThreads = QG_SQ_THREADS;
constexpr int kSqMinCtas = 65536 / (kSqThreads * QG_SQ_MAXREG);
static_assert(kSqThreads >= 128, "one thread per multiplier-table entry");
// Blocks whose loads are in flight together in one thread.
template <bool kBf16>
constexpr int kSqUnroll = kBf16 ? 2 : 1;

template <bool kBf16>
__global__ void __launch_bounds__(kSqThreads, kSqMinCtas) skinny_amax_kernel(const __grid_constant__ SkinnyParams p) {
  griddep_launch_dependents();
  if (kDiag & 64u) {
    if (threadIdx.x == 0 && blockIdx.x == (kDiag >> 16)) {
      auto* tr = reinterpret_cast<unsigned long long*>(p.part + static_cast<int64_t>(kSkinnyMaxCtas - 1) * p.slices * p.m * 128);
      tr[506] = tr[1];  // the previous call's GEMM end
    }
    if (threadIdx.x == 0) trace(p, 500);
  }
  const int G = gridDim.x, c = blockIdx.x;
  const int64_t nblocks = static_cast<int64_t>(p.m) * (p.k / 16);
  const int64_t b0 = nblocks * c / G, b1 = nblocks * (c + 1) / G;
  constexpr int kU = kSqUnroll<kBf16>;
  float mx = 0.0f;
  for (int64_t b = b0 + threadIdx.x; b < b1; b += kU * kSqThreads) {
    RawBlock<kBf16> r[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (b + u * kSqThreads < b1) r[u].load(p.x, b + u * kSqThreads);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (b + u * kSqThreads >= b1) break;
      float v[16];
      r[u].decode(v);
#pragma unroll
      for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __shared__ float red[kSqThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = red[0];
    for (int w = 1; w < kSqThreads / 32; ++w) a = fmaxf(a, red[w]);
    p.amax_part[c] = a;
    trace(p, 501);
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(kSqThreads, kSqMinCtas)
    skinny_quant_kernel(const __grid_constant__ SkinnyParams p, int amax_ctas) {
  griddep_launch_dependents();
  const int G = gridDim.x, c = blockIdx.x;
  const int64_t sfk = p.k / 16;
  const int64_t nblocks = static_cast<int64_t>(p.m) * sfk;
  const int64_t b0 = nblocks * c / G, b1 = nblocks * (c + 1) / G;
  constexpr int kU = kSqUnroll<kBf16>;
  RawBlock<kBf16> r[kU];
  auto load_batch = [&](int64_t b) {
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (b + u * kSqThreads < b1) r[u].load(p.x, b + u * kSqThreads);
  };
  // x is ready before the amax kernel starts (an ordinary launch, after the
  // stream's previous kernel): the first blocks are loaded before waiting
  // for it.
  if (threadIdx.x == 0) trace(p, 502);
  load_batch(b0 + threadIdx.x);
  griddep_wait();  // every amax partial is written
  if (threadIdx.x == 0) trace(p, 503);
  float a = 0.0f;
  for (int r = threadIdx.x; r < amax_ctas; r += kSqThreads) a = fmaxf(a, __ldcg(p.amax_part + r));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  __shared__ float red[kSqThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  float amax = red[0];
  for (int w = 1; w < kSqThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float ts = amax > 0.0f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  const float inv_ts = __fdiv_rn(1.0f, ts);
  // mult[c] = inv_ts / e4m3(c), the element multiplier of a block whose
  // scale code is c (0 for the zero code), as the per-block division has it.
  __shared__ float mult_tab[128];
  if (threadIdx.x < 128) {
    const float bs = e4m3_decode_positive(threadIdx.x);
    mult_tab[threadIdx.x] = bs > 0.0f ? __fdiv_rn(inv_ts, bs) : 0.0f;
  }
  __syncthreads();
  if (threadIdx.x == 0) trace(p, 505);
  if (c == 0 && threadIdx.x == 0) *p.x_ts = ts;
  const int64_t sf_blocks = (sfk + 3) / 4;  // one 128-row block: m <= 128
  const bool idx32 = nblocks <= 0xffffffffll;
  for (int64_t b = b0 + threadIdx.x; b < b1; b += kU * kSqThreads) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t bu = b + u * kSqThreads;
      if (bu >= b1) break;
      float v[16];
      r[u].decode(v);
      float bmax = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
      const uint32_t sbits = e4m3_round_up(__fdiv_rn(__fmul_rn(bmax, inv_ts), 6.0f));
      const float mult = mult_tab[sbits];
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        float x0 = __fmul_rn(v[i], mult), x1 = __fmul_rn(v[i + 1], mult);
        x0 = x0 == x0 ? x0 : 0.0f;  // NaN -> +0
        x1 = x1 == x1 ? x1 : 0.0f;
        const uint32_t byte = e2m1x2_cvt(x1, x0);
        if (i < 8) lo |= byte << (4 * i);
        else hi |= byte << (4 * (i - 8));
      }
      reinterpret_cast<uint2*>(p.xq)[bu] = make_uint2(lo, hi);
      const int64_t row = idx32 ? static_cast<int64_t>(static_cast<uint32_t>(bu) /
                                                       static_cast<uint32_t>(sfk))
                                : bu / sfk;
      const int64_t sc = bu - row * sfk;
      p.xsf[mma_scale_offset(row, sc, 1, sf_blocks, 1)] = static_cast<uint8_t>(sbits);
    }
    load_batch(b + kU * kSqThreads);
  }
  // Padding scale slots (rows >= m, scale columns >= k/16) read as zero, and
  // the GEMM's split-tile counters start at zero.
  const int64_t cols_pad = sf_blocks * 4, npad = 128 * cols_pad;
  const int64_t gt = static_cast<int64_t>(c) * kSqThreads + threadIdx.x;
  const int64_t gstride = static_cast<int64_t>(G) * kSqThreads;
  if (sfk % 4 == 0) {
    // Whole padding rows: one 32-bit word holds a row's four scales of a
    // 512-byte chunk.
    const int64_t prow = 128 - p.m, nwords = prow * sf_blocks;
    uint32_t* w = reinterpret_cast<uint32_t*>(p.xsf);
    for (int64_t i = gt; i < nwords; i += gstride) {
      const int64_t chunk = i / prow, row = p.m + (i - chunk * prow);
      w[chunk * 128 + (row & 31) * 4 + (row >> 5)] = 0u;
    }
  } else if (npad != nblocks) {
    for (int64_t i = gt; i < npad; i += gstride) {
      const int64_t row = i / cols_pad, sc = i - row * cols_pad;
      if (row >= p.m || sc >= sfk) p.xsf[mma_scale_offset(row, sc, 1, sf_blocks, 1)] = 0u;
    }
  }
  for (int64_t i = gt; i < static_cast<int64_t>(p.num_counters); i += gstride) p.cnt[i] = 0u;
  if (threadIdx.x == 0) trace(p, 504);
}

template <int kN>
__global__ void QG_SKINNY_BOUNDS gemm_skinny_kernel(const __grid_constant__ SkinnyParams p) {
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
  if (threadIdx.x == 0) trace_cta(p, 768 + blockIdx.x);
  UnitRange ur;
  ur.init(p.num_tiles, p.num_k_blocks, static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x));
  // Every role but the weight producer waits for the quantiser kernels
  // here, before any bounded wait starts its clock.
  if (warp != 0) griddep_wait();

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
      // loads wait for the quantiser kernels (griddepcontrol.wait), so the
      // weight stream runs while the activations are being quantised.
      // 128-row tiles: a rolling lead of kL2Ahead units ahead of the stage
      // ring (prefetched as each stage is issued); wide tiles: kL2Ahead
      // units once, when the activation loads are released.  Swept on one
      // box (GB/s, m = 16 / 64 / 128): no rolling lead, 8 units: 5185 /
      // 4241 / 4299; rolling 1: 5595 / 4366 / 4275; rolling 2: 5580 / 4335 /
      // 4067; rolling 4: 5355 / 4200 / 4063; rolling 8: 4770 / 3631 / 3911.
      // A deeper lead competes with the ring's own loads for the same HBM.
      constexpr bool kL2Roll = Cfg::kH == 1 ? QG_SKINNY_L2_ROLL : QG_SKINNY_L2_ROLL_WIDE;
      constexpr int kL2Ahead = Cfg::kH == 1 ? QG_SKINNY_L2_AHEAD : QG_SKINNY_L2_AHEAD_WIDE;  // units (32 KB of weights each)
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
      auto prefetch_unit = [&](const SegCursor& u) {
#pragma unroll
        for (int hf = 0; hf < Cfg::kH; ++hf) {
          const int rb = u.t * Cfg::kH + hf;  // 128-row block
          tma_prefetch_l2_3d(&p.tm_sfw, 0, rb, u.kb * Cfg::kSfChunks);
#pragma unroll
          for (int h = 0; h < Cfg::kBoxes; ++h)
            tma_prefetch_l2_2d(&p.tm_w, u.kb * Cfg::kBKBytes + h * Cfg::kBoxBytes,
                               rb * Cfg::kBM);
        }
      };
      SegCursor pf;
      bool pf_more = false;
      auto release_deferred = [&](SegCursor ahead, bool more) {
        for (int i = 0; more && i < kL2Ahead; ++i) {
          prefetch_unit(ahead);
          more = ahead.next();
        }
        pf = ahead;
        pf_more = more;
        griddep_wait();  // the quantiser kernels have written xq / xsf
        asm volatile("fence.proxy.async.global;" ::: "memory");  // read by TMA
        trace(p, 2);
        trace_cta(p, 1024 + blockIdx.x);
        for (int s = 0; s < deferred; ++s) issue_x(s, dkb[s]);
        dep_done = true;
      };
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
#pragma unroll
        for (int hf = 0; hf < Cfg::kH; ++hf) {
          const int rb = cur.t * Cfg::kH + hf;  // 128-row block
          tma_load_3d(ssfw + hf * Cfg::kSfChunks * 512, &p.tm_sfw, &full_bar[stage], 0, rb,
                      cur.kb * Cfg::kSfChunks, pol_w);
#pragma unroll
          for (int h = 0; h < Cfg::kBoxes; ++h)
            tma_load_2d(sw + (h * Cfg::kH + hf) * Cfg::kWBox, &p.tm_w, &full_bar[stage],
                        cur.kb * Cfg::kBKBytes + h * Cfg::kBoxBytes, rb * Cfg::kBM, pol_w);
        }
        if (dep_done) {
          issue_x(stage, cur.kb);
          if (kL2Roll && pf_more) {  // keep kL2Ahead units in L2 ahead
            prefetch_unit(pf);
            pf_more = pf.next();
          }
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
        const int buf = seg % Cfg::kAccBufs;
        if (!mbar_wait_bounded(&acc_empty[buf], ((seg / Cfg::kAccBufs) & 1) ^ 1u, p.timeout_ns,
                               abort_flag, p.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * Cfg::kH * kN);
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
            // MMA i: half hf = i / kSfChunks, chunk c (box c / 4, 32-byte K
            // step c % 4 inside the 128-byte row).
            const int hf = i / Cfg::kSfChunks, c = i % Cfg::kSfChunks;
            const uint64_t wo = static_cast<uint64_t>(((c / 4) * Cfg::kH + hf) * (Cfg::kWBox >> 4) +
                                                      (c % 4) * 2);
            const uint64_t xo = static_cast<uint64_t>((c / 4) * (Cfg::kXBox >> 4) + (c % 4) * 2);
            mma_mxf4nvf4(d_tmem + static_cast<uint32_t>(hf * kN), wdesc + wo, xdesc + xo, idesc,
                         sfw_col + hf * 4 * Cfg::kSfChunks + c * 4,
                         sfw_col + Cfg::kH * 4 * Cfg::kSfChunks + c * 4, (acc | c) != 0 ? 1u : 0u);
          }
          acc = 1;
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
    for (int u = 0; u < my_units; ++u) {
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded(&full_bar[stage], phase, p.timeout_ns, abort_flag, p.status,
                               kDevTimeoutMma);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(&full_bar[stage], phase);
      const uint8_t* ssfw = smem + stage * Cfg::kStageBytes + Cfg::kWBytes + Cfg::kXBytes;
      const uint8_t* ssfx = ssfw + Cfg::kSfwBytes;
      // The weight scales of each half, then the activation scales (4
      // columns per 64-K chunk each) in the stage's slot, written with ONE
      // tcgen05.st (a store costs about the same whatever its width).
      uint32_t v[Cfg::kSfStageCols];
#pragma unroll
      for (int j = 0; j < Cfg::kH + 1; ++j)
#pragma unroll
        for (int c = 0; c < Cfg::kSfChunks; ++c) {
          const uint4 x = lds128((j < Cfg::kH ? ssfw + j * Cfg::kSfChunks * 512 : ssfx) + c * 512 +
                                 lane * 16);
          uint32_t* d = v + (j * Cfg::kSfChunks + c) * 4;
          d[0] = x.x; d[1] = x.y; d[2] = x.z; d[3] = x.w;
        }
#pragma unroll
      for (int j = Cfg::kSfWords; j < Cfg::kSfStageCols; ++j) v[j] = 0u;
      const uint32_t col = Cfg::kTmemSfBase + stage * Cfg::kSfStageCols;
      if (!(kDiag & 1u)) {
        tmem_st_32x32b<Cfg::kSfStageCols>(t_quad + col, v);
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
    griddep_wait();  // the activation tensor scale and the tile counters
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
    for (int seg = 0; seg < order.nseg(); ++seg) {
      const int t = order.tile_of(seg);
      const int buf = seg % Cfg::kAccBufs;
      const uint32_t par = static_cast<uint32_t>(seg / Cfg::kAccBufs) & 1u;
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded<false, 128>(&acc_full[buf], par, p.timeout_ns, abort_flag,
                                           p.status, kDevTimeoutEpilogue);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      mbar_try_wait(&acc_full[buf], par);
      tc_fence_after();
      if (quad == 0 && lane == 0) trace(p, 120 + seg);
      if (quad == 0 && lane == 0 && seg == order.nseg() - 1) trace_cta(p, 1536 + blockIdx.x);
      // Contributors of a split tile (whole tiles: this CTA alone).
      const bool split = order.split(seg);
      const int cf = split ? ur.contributor(static_cast<int64_t>(t) * ur.nkb, grid)
                           : static_cast<int>(blockIdx.x);
      const int cl = split ? ur.contributor(static_cast<int64_t>(t + 1) * ur.nkb - 1, grid)
                           : static_cast<int>(blockIdx.x);
      // Each 128-row half of the tile is stored, counted and summed as a
      // tile of its own (vt: its 128-row block; its counter and slices):
      // first both halves' stores, then both halves' counting.
#pragma unroll 1
      for (int hf = 0; hf < Cfg::kH; ++hf) {
      const int vt = t * Cfg::kH + hf;
      const int col = quad * 32 + lane;
      const int n = vt * Cfg::kBM + col;
      const bool n_ok = n < p.n;
      float* mine = p.part + (static_cast<int64_t>(blockIdx.x * 2 + (t == my_first ? 0 : 1)) *
                                  Cfg::kH + hf) * p.m * Cfg::kBM;
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
      const int n_tail = vt * Cfg::kBM + quad * 32;
      const bool bf16_tail = bf16_dst && seg == order.nseg() - 1 && p.vec_ok && n_tail + 32 <= p.n;
#pragma unroll
      for (int gc = 0; gc < kN / kGroup; ++gc) {
        uint32_t r[kGroup];
#pragma unroll
        for (int cc = 0; cc < kGroup / 16; ++cc)
          tmem_ld_32x32b_x16(t_quad + static_cast<uint32_t>((buf * Cfg::kH + hf) * kN +
                                                            gc * kGroup + cc * 16),
                             *reinterpret_cast<uint32_t(*)[16]>(r + cc * 16));
        tmem_wait_ld();
        if (gc == kN / kGroup - 1 && hf == Cfg::kH - 1) {
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
      }  // halves: stores
      if (cf == cl) continue;
      // The accumulator is released (after the last half's reads) before
      // any counting or summing, so the next segment's MMAs do not wait for
      // a sum pass.
#pragma unroll 1
      for (int hf = 0; hf < Cfg::kH; ++hf) {
      const int vt = t * Cfg::kH + hf;
      // Publish the slice and count this contributor with one acquire-release
      // atomic from lane 0: the warp barrier before it orders every lane's
      // slice stores ahead of the release (fence cumulativity), the one after
      // it orders every lane's slice reads behind the acquire.  Two full
      // fences here each cost ~2 us while the weight stream loads the memory
      // system.
      if (quad == 0 && lane == 0) trace(p, 300 + 4 * seg);
      __syncwarp();
      uint32_t old = 0;
      if (lane == 0) old = atom_add_acq_rel_gpu(&p.cnt[vt * 4 + quad], 1u);
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
        const int nb = vt * Cfg::kBM + quad * 32 + c8;
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
            auto slice_of = [&](int cc) {
              return p.part + ((cc * 2 + (t == first_tile(cc) ? 0 : 1)) * Cfg::kH + hf) * slice +
                     quad * 32 + c8;
            };
            const float* s0 = slice_of(c);
            const float* s1 = two ? slice_of(c + 1) : s0;
            const float* s2 = three ? slice_of(c + 2) : s0;
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
      if (lane == 0) p.cnt[vt * 4 + quad] = 0u;  // ready for the next call
      if (quad == 0 && lane == 0) trace_cta(p, 1280 + blockIdx.x);
      if (quad == 0 && lane == 0) trace(p, 200 + seg);
      }  // halves: counting and sums
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
  // Programmatic dependent launch: the CTAs start (and stream weights) while
  // the quantiser kernel ahead of it still runs; griddepcontrol.wait in the
  // producer and the epilogue orders what they read after it.
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// The two quantiser kernels of a call (see skinny_quant_kernel): the amax
// pass is ordered after the stream's earlier work as usual (the activations
// may come from it), the quantising pass launches early and waits for it.
cudaError_t launch_skinny_quant(const SkinnyParams& p, int grid, cudaStream_t stream) {
  // An SM changes its shared-memory carveout only when it is idle: the small
  // kernels ask for the full carveout the GEMM runs with, so that a GEMM CTA
  // can join them on the SM instead of waiting for them to drain.
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    const void* fns[4] = {reinterpret_cast<const void*>(skinny_amax_kernel<true>),
                          reinterpret_cast<const void*>(skinny_amax_kernel<false>),
                          reinterpret_cast<const void*>(skinny_quant_kernel<true>),
                          reinterpret_cast<const void*>(skinny_quant_kernel<false>)};
    for (const void* f : fns) {
      cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout,
                                           cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return e;
    }
    attr_done[dev] = true;
  }
  if (p.x_bf16) skinny_amax_kernel<true><<<grid, kSqThreads, 0, stream>>>(p);
  else skinny_amax_kernel<false><<<grid, kSqThreads, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kSqThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return p.x_bf16 ? cudaLaunchKernelEx(&cfg, skinny_quant_kernel<true>, p, grid)
                  : cudaLaunchKernelEx(&cfg, skinny_quant_kernel<false>, p, grid);
}

int skinny_quant_grid(int64_t xblocks, int sms) {
  int64_t g = (xblocks + kSqThreads - 1) / kSqThreads;  // one block per thread
  if (g > sms) g = sms;
  return g < 1 ? 1 : static_cast<int>(g);
}

template <int kN>
static SkinnyShape shape_of() {
  using Cfg = SkinnyCfg<kN>;
  SkinnyShape sh;
  sh.tile_rows = Cfg::kTileRows;
  sh.stage_k_bytes = Cfg::kBKBytes;
  sh.sf_chunks = Cfg::kSfChunks;
  sh.halves = Cfg::kH;
  return sh;
}

SkinnyShape skinny_shape(int64_t m) {
  switch (skinny_mma_n(m)) {
    case 16: return shape_of<16>();
    case 32: return shape_of<32>();
    case 64: return shape_of<64>();
    default: return shape_of<128>();
  }
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
