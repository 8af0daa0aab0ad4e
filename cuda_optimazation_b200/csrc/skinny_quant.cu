// skinny_quant.cu -- one-launch NVFP4 activation quantizer for the decode
// GEMM (m <= 128 rows).
//
// The two-pass quantizer in quantize.cu needs a zeroed amax word, an amax
// grid and a quantize grid: three dependent launches whose gaps dominate at
// decode sizes (m * k <= 1 Mi elements).  Here one thread-block cluster does
// the whole job: every CTA takes a contiguous range of 16-element blocks,
// reduces its amax, the CTAs exchange their maxima through distributed
// shared memory, and each CTA then quantises its own range (a second read,
// served by L2).  The arithmetic is make_nvfp4_reference's
// (GEMMsm110/include/requant/nvfp4_reference.cuh:76-112), bit for bit, with
// the same codecs as quantize.cu.
//
// The kernel also zeroes the GEMM's per-tile arrival counters and lets the
// GEMM grid launch early (programmatic dependent launch): the GEMM waits on
// this grid only where it reads what it writes.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "qg_codec.cuh"
#include "qg_gemm.h"
#include "qg_ptx.cuh"

namespace qg {

namespace cg = cooperative_groups;

constexpr int kQCluster = 8;
constexpr int kQThreads = 1024;

// Raw 16-element block (bf16: 32 bytes, fp32: 64 bytes) so several blocks'
// loads can be in flight per thread before any is decoded.
template <bool kBf16>
struct RawBlock {
  uint4 w[kBf16 ? 2 : 4];
  __device__ __forceinline__ void load(const void* x, int64_t blk) {
    const uint4* p = reinterpret_cast<const uint4*>(x) + blk * (kBf16 ? 2 : 4);
#pragma unroll
    for (int i = 0; i < (kBf16 ? 2 : 4); ++i) w[i] = __ldg(p + i);
  }
  __device__ __forceinline__ void decode(float (&v)[16]) const {
#pragma unroll
    for (int i = 0; i < (kBf16 ? 2 : 4); ++i) {
      const uint32_t u[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (kBf16) {
          v[8 * i + 2 * j] = __uint_as_float(u[j] << 16);
          v[8 * i + 2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
        } else {
          v[4 * i + j] = __uint_as_float(u[j]);
        }
      }
    }
  }
};

template <bool kBf16>
__global__ void __cluster_dims__(kQCluster, 1, 1) __launch_bounds__(kQThreads)
    skinny_quantize_kernel(const void* x, int64_t m, int64_t k, uint8_t* q, uint8_t* sf,
                           float* ts_out, uint32_t* cnt, int64_t ncnt) {
  griddep_launch_dependents();
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float red[kQThreads / 32];
  __shared__ float cta_amax;
  const int rank = static_cast<int>(cluster.block_rank());
  const int tid = threadIdx.x;
  const int64_t sfk = k / 16;
  const int64_t nblocks = m * sfk;
  const int64_t b0 = nblocks * rank / kQCluster;
  const int64_t b1 = nblocks * (rank + 1) / kQCluster;

  for (int64_t i = static_cast<int64_t>(rank) * kQThreads + tid; i < ncnt;
       i += kQCluster * kQThreads)
    cnt[i] = 0u;

  // ---- pass 1: amax of this CTA's blocks, then of the cluster
  constexpr int kFly = kBf16 ? 4 : 2;  // blocks in flight per thread
  float mx = 0.0f;
  for (int64_t base = b0 + tid; base < b1; base += kFly * kQThreads) {
    RawBlock<kBf16> r[kFly];
#pragma unroll
    for (int f = 0; f < kFly; ++f)
      if (base + f * kQThreads < b1) r[f].load(x, base + f * kQThreads);
#pragma unroll
    for (int f = 0; f < kFly; ++f) {
      if (base + f * kQThreads >= b1) break;
      float v[16];
      r[f].decode(v);
#pragma unroll
      for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid < 32) {
    mx = tid < kQThreads / 32 ? red[tid] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (tid == 0) cta_amax = mx;
  }
  cluster.sync();
  float amax = 0.0f;
#pragma unroll
  for (int r = 0; r < kQCluster; ++r) amax = fmaxf(amax, *cluster.map_shared_rank(&cta_amax, r));
  cluster.sync();  // peers' shared memory stays live until every CTA has read it

  const float ts = amax > 0.0f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  const float inv_ts = __fdiv_rn(1.0f, ts);
  if (rank == 0 && tid == 0) *ts_out = ts;

  // ---- pass 2: quantise (MMA layout: low nibble first, chunked scales)
  const int64_t row_blocks = (m + 127) / 128;
  const int64_t sf_blocks = (sfk + 3) / 4;
  for (int64_t base = b0 + tid; base < b1; base += kFly * kQThreads) {
    RawBlock<kBf16> r[kFly];
#pragma unroll
    for (int f = 0; f < kFly; ++f)
      if (base + f * kQThreads < b1) r[f].load(x, base + f * kQThreads);
#pragma unroll
    for (int f = 0; f < kFly; ++f) {
      const int64_t b = base + f * kQThreads;
      if (b >= b1) break;
      float v[16];
      r[f].decode(v);
      float bmax = 0.0f;
  #pragma unroll
      for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
      const float namax = __fmul_rn(bmax, inv_ts);
      const uint32_t sbits = e4m3_round_up(__fdiv_rn(namax, 6.0f));
      const float bs = e4m3_decode_positive(sbits);
      const float mult = bs > 0.0f ? __fdiv_rn(inv_ts, bs) : 0.0f;
      uint32_t lo = 0, hi = 0;
  #pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const uint32_t byte = e2m1_encode(__fmul_rn(v[i], mult)) |
                              (e2m1_encode(__fmul_rn(v[i + 1], mult)) << 4);
        if (i < 8) lo |= byte << (4 * i);
        else hi |= byte << (4 * (i - 8));
      }
      reinterpret_cast<uint2*>(q)[b] = make_uint2(lo, hi);
      const int64_t row = b / sfk, sc = b - row * sfk;
      sf[mma_scale_offset(row, sc, row_blocks, sf_blocks, 1)] = static_cast<uint8_t>(sbits);
    }
  }

  // ---- padding scale slots (rows >= m, scale columns >= k/16) read as 0
  const int64_t rows_pad = row_blocks * 128, cols_pad = sf_blocks * 4;
  const int64_t npad = rows_pad * cols_pad;
  if (npad != nblocks) {
    for (int64_t i = static_cast<int64_t>(rank) * kQThreads + tid; i < npad;
         i += kQCluster * kQThreads) {
      const int64_t row = i / cols_pad, sc = i - row * cols_pad;
      if (row >= m || sc >= sfk) sf[mma_scale_offset(row, sc, row_blocks, sf_blocks, 1)] = 0u;
    }
  }
}

cudaError_t launch_skinny_quantize(const void* x, bool bf16, int64_t m, int64_t k, uint8_t* q,
                                   uint8_t* sf, float* ts, uint32_t* cnt, int64_t ncnt,
                                   cudaStream_t stream) {
  if (bf16)
    skinny_quantize_kernel<true><<<kQCluster, kQThreads, 0, stream>>>(x, m, k, q, sf, ts, cnt, ncnt);
  else
    skinny_quantize_kernel<false><<<kQCluster, kQThreads, 0, stream>>>(x, m, k, q, sf, ts, cnt,
                                                                       ncnt);
  return cudaGetLastError();
}

}  // namespace qg
