// quantize.cu -- NVFP4 / MXFP8 activation quantizers, the NVFP4 layout
// repack, and the bounded-wait self test.
//
// NVFP4 follows make_nvfp4_reference
// (GEMMsm110/include/requant/nvfp4_reference.cuh:76-112) bit for bit:
//   ts      = amax / (448 * 6)            (1 if amax == 0)
//   s_blk   = e4m3_round_up(max|x * (1/ts)| / 6)
//   mult    = (1/ts) / decode(s_blk)      (0 if the scale decodes to 0)
//   q_i     = e2m1_rne(x_i * mult)
// Every step uses IEEE round-to-nearest fp32 operations (__fdiv_rn /
// __fmul_rn) so the device result equals the host reference exactly; the
// reference's own device twin used inv_ts * (1/s) instead
// (sm110_tcgen05_epilogue.cuh:148-150), which is not bit-identical.
//
// The work is HBM-bound (4 or 2 bytes in, 0.5625 out per element): loads are
// 16-byte vectors, one thread per 16-element block, grid sized in multiples
// of the SM count.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "qg_gemm.h"
#include "qg_ptx.cuh"
#include "qg_codec.cuh"

namespace qg {

// ------------------------------------------------------------------ amax
template <bool kBf16>
__global__ void __launch_bounds__(256) amax_kernel(const void* x, int64_t n, uint32_t* amax_bits) {
  float m = 0.0f;
  const int64_t nvec = n / 16;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < nvec;
       v += stride) {
    float f[16];
    load16<kBf16>(x, v * 16, f);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(f[i]));
  }
  for (int64_t i = nvec * 16 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += stride)
    m = fmaxf(m, fabsf(load1<kBf16>(x, i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // Non-negative floats order like their bit patterns.
    if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m));
  }
}

// ------------------------------------------------------------------ NVFP4
// One thread per 16-element block.  layout: 0 REF_LINEAR (flat blocks, high
// nibble first, linear scales), 1 MMA, 2 MMA_KMAJOR (row blocks, low nibble
// first, chunked scales).
template <bool kBf16>
__global__ void __launch_bounds__(256)
    nvfp4_quantize_kernel(const void* x, int64_t rows, int64_t k, int layout, uint8_t* q,
                          uint8_t* sf, float* ts_out, const uint32_t* amax_bits) {
  const float amax = __uint_as_float(*amax_bits);
  const float ts = amax > 0.0f ? __fdiv_rn(amax, 2688.0f) : 1.0f;
  const float inv_ts = __fdiv_rn(1.0f, ts);
  const int64_t n = rows * k;
  const int64_t nblocks = (n + 15) / 16;
  const int64_t sfk = k / 16;
  const int64_t row_blocks = (rows + 127) / 128;
  const int64_t sf_blocks = (sfk + 3) / 4;
  if (blockIdx.x == 0 && threadIdx.x == 0 && ts_out) *ts_out = ts;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += stride) {
    float v[16];
    if ((b + 1) * 16 <= n) {
      load16<kBf16>(x, b * 16, v);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = (b * 16 + i < n) ? load1<kBf16>(x, b * 16 + i) : 0.0f;
    }
    float bmax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
    // max|x*inv_ts| == RN(max|x| * inv_ts): RN is monotonic.
    const float namax = __fmul_rn(bmax, inv_ts);
    const uint32_t sbits = e4m3_round_up(__fdiv_rn(namax, 6.0f));
    const float bs = e4m3_decode_positive(sbits);
    const float mult = bs > 0.0f ? __fdiv_rn(inv_ts, bs) : 0.0f;
    uint32_t lo = 0, hi = 0;
    const bool high_first = (layout == 0);
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const uint32_t c0 = e2m1_encode(__fmul_rn(v[i], mult));
      const uint32_t c1 = e2m1_encode(__fmul_rn(v[i + 1], mult));
      const uint32_t byte = high_first ? ((c0 << 4) | c1) : (c0 | (c1 << 4));
      if (i < 8) lo |= byte << (4 * i);
      else hi |= byte << (4 * (i - 8));
    }
    reinterpret_cast<uint2*>(q)[b] = make_uint2(lo, hi);
    if (layout == 0) {
      sf[b] = static_cast<uint8_t>(sbits);
    } else {
      const int64_t row = b / sfk, sc = b - row * sfk;
      sf[mma_scale_offset(row, sc, row_blocks, sf_blocks, layout)] = static_cast<uint8_t>(sbits);
    }
  }
}

// ------------------------------------------------------------------ MXFP8
// One thread per 32-element block: ue8m0 exponent floor(log2(amax)) - 8,
// elements RN-satfinite e4m3 of x * 2^-e.
__device__ __forceinline__ int floor_log2_positive(float a) {
  const uint32_t b = __float_as_uint(a);
  const int e = static_cast<int>((b >> 23) & 0xffu);
  if (e != 0) return e - 127;
  return -149 + (31 - __clz(static_cast<int>(b & 0x7fffffu)));
}

__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <bool kBf16>
__global__ void __launch_bounds__(256)
    mxfp8_quantize_kernel(const void* x, int64_t rows, int64_t k, int layout, uint8_t* q,
                          uint8_t* sf) {
  const int64_t sfk = k / 32;
  const int64_t nblocks = rows * sfk;
  const int64_t row_blocks = (rows + 127) / 128;
  const int64_t sf_blocks = (sfk + 3) / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += stride) {
    float v[32];
    load16<kBf16>(x, b * 32, *reinterpret_cast<float(*)[16]>(&v[0]));
    load16<kBf16>(x, b * 32 + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    int e = -127;
    if (amax > 0.0f) e = max(-127, min(127, floor_log2_positive(amax) - 8));
    const float mul = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e, normal
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t p0 = cvt_e4m3x2(__fmul_rn(v[4 * i], mul), __fmul_rn(v[4 * i + 1], mul));
      const uint32_t p1 = cvt_e4m3x2(__fmul_rn(v[4 * i + 2], mul), __fmul_rn(v[4 * i + 3], mul));
      w[i] = p0 | (p1 << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(q + b * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    const uint8_t code = static_cast<uint8_t>(e + 127);
    if (layout == 0) {
      sf[b] = code;
    } else {
      const int64_t row = b / sfk, sc = b - row * sfk;
      sf[mma_scale_offset(row, sc, row_blocks, sf_blocks, layout)] = code;
    }
  }
}

// ------------------------------------------------------------------ MXFP4
// OCP MX v1.0 with E2M1 elements: one thread per 32-element block, ue8m0
// exponent e = floor(log2(amax)) - 2 (emax of E2M1) clamped to [-127, 127]
// (all-zero block: code 0), elements e2m1 RNE, saturating, of x * 2^-e
// (NaN -> +0).  layout 0 packs the first element of a pair in the high
// nibble, the MMA layouts in the low nibble.
template <bool kBf16>
__global__ void __launch_bounds__(256)
    mxfp4_quantize_kernel(const void* x, int64_t rows, int64_t k, int layout, uint8_t* q,
                          uint8_t* sf) {
  const int64_t sfk = k / 32;
  const int64_t nblocks = rows * sfk;
  const int64_t row_blocks = (rows + 127) / 128;
  const int64_t sf_blocks = (sfk + 3) / 4;
  const bool high_first = layout == 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += stride) {
    float v[32];
    load16<kBf16>(x, b * 32, *reinterpret_cast<float(*)[16]>(&v[0]));
    load16<kBf16>(x, b * 32 + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    int e = -127;
    if (amax > 0.0f) e = max(-127, min(127, floor_log2_positive(amax) - 2));
    // 2^-e: e <= 125 here, so the exponent field 127 - e is in [2, 254].
    const float mul = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float x0 = __fmul_rn(v[8 * i + 2 * j], mul), x1 = __fmul_rn(v[8 * i + 2 * j + 1], mul);
        x0 = x0 == x0 ? x0 : 0.0f;  // NaN -> +0
        x1 = x1 == x1 ? x1 : 0.0f;
        word |= (high_first ? e2m1x2_cvt(x0, x1) : e2m1x2_cvt(x1, x0)) << (8 * j);
      }
      w[i] = word;
    }
    reinterpret_cast<uint4*>(q)[b] = make_uint4(w[0], w[1], w[2], w[3]);
    const uint8_t code = static_cast<uint8_t>(e + 127);
    if (layout == 0) {
      sf[b] = code;
    } else {
      const int64_t row = b / sfk, sc = b - row * sfk;
      sf[mma_scale_offset(row, sc, row_blocks, sf_blocks, layout)] = code;
    }
  }
}

// ------------------------------------------------------------------ repack
__global__ void __launch_bounds__(256)
    nvfp4_repack_kernel(const uint8_t* sq, const uint8_t* ssf, int src_layout, uint8_t* dq,
                        uint8_t* dsf, int dst_layout, int64_t rows, int64_t k) {
  const int64_t sfk = k / 16;
  const int64_t nblocks = rows * sfk;
  const int64_t row_blocks = (rows + 127) / 128;
  const int64_t sf_blocks = (sfk + 3) / 4;
  const bool swap = (src_layout == 0) != (dst_layout == 0);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += stride) {
    uint2 w = reinterpret_cast<const uint2*>(sq)[b];
    if (swap) {
      w.x = ((w.x >> 4) & 0x0f0f0f0fu) | ((w.x << 4) & 0xf0f0f0f0u);
      w.y = ((w.y >> 4) & 0x0f0f0f0fu) | ((w.y << 4) & 0xf0f0f0f0u);
    }
    reinterpret_cast<uint2*>(dq)[b] = w;
    const int64_t row = b / sfk, sc = b - row * sfk;
    const int64_t so =
        src_layout == 0 ? b : mma_scale_offset(row, sc, row_blocks, sf_blocks, src_layout);
    const int64_t d =
        dst_layout == 0 ? b : mma_scale_offset(row, sc, row_blocks, sf_blocks, dst_layout);
    dsf[d] = ssf[so];
  }
}

// MX formats (one ue8m0 scale per 32 K elements): a block is 16 value bytes
// (MXFP4, nibble order flipped between REF_LINEAR and the MMA layouts) or 32
// (MXFP8, bytes unchanged); one thread per block.
template <bool kFp4>
__global__ void __launch_bounds__(256)
    mx_repack_kernel(const uint8_t* sq, const uint8_t* ssf, int src_layout, uint8_t* dq,
                     uint8_t* dsf, int dst_layout, int64_t rows, int64_t k) {
  constexpr int kVec = kFp4 ? 1 : 2;  // uint4 per block
  const int64_t sfk = k / 32;
  const int64_t nblocks = rows * sfk;
  const int64_t row_blocks = (rows + 127) / 128;
  const int64_t sf_blocks = (sfk + 3) / 4;
  const bool swap = kFp4 && ((src_layout == 0) != (dst_layout == 0));
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += stride) {
#pragma unroll
    for (int v = 0; v < kVec; ++v) {
      uint4 w = reinterpret_cast<const uint4*>(sq)[b * kVec + v];
      if (swap) {
        w.x = ((w.x >> 4) & 0x0f0f0f0fu) | ((w.x << 4) & 0xf0f0f0f0u);
        w.y = ((w.y >> 4) & 0x0f0f0f0fu) | ((w.y << 4) & 0xf0f0f0f0u);
        w.z = ((w.z >> 4) & 0x0f0f0f0fu) | ((w.z << 4) & 0xf0f0f0f0u);
        w.w = ((w.w >> 4) & 0x0f0f0f0fu) | ((w.w << 4) & 0xf0f0f0f0u);
      }
      reinterpret_cast<uint4*>(dq)[b * kVec + v] = w;
    }
    const int64_t row = b / sfk, sc = b - row * sfk;
    const int64_t so =
        src_layout == 0 ? b : mma_scale_offset(row, sc, row_blocks, sf_blocks, src_layout);
    const int64_t d =
        dst_layout == 0 ? b : mma_scale_offset(row, sc, row_blocks, sf_blocks, dst_layout);
    dsf[d] = ssf[so];
  }
}

static int grid_for(int64_t work_items, int threads);

cudaError_t launch_repack_mx(bool fp4, const uint8_t* sq, const uint8_t* ssf, int src_layout,
                             uint8_t* dq, uint8_t* dsf, int dst_layout, int64_t rows, int64_t k,
                             cudaStream_t stream) {
  const int grid = grid_for(rows * (k / 32), 256);
  if (fp4)
    mx_repack_kernel<true><<<grid, 256, 0, stream>>>(sq, ssf, src_layout, dq, dsf, dst_layout,
                                                     rows, k);
  else
    mx_repack_kernel<false><<<grid, 256, 0, stream>>>(sq, ssf, src_layout, dq, dsf, dst_layout,
                                                      rows, k);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ self test
__global__ void wait_timeout_selftest_kernel(uint64_t timeout_ns, uint32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0u;
    fence_barrier_init();
    // Nobody arrives: phase 0 never completes, the bounded wait must expire.
    mbar_wait_bounded(&bar, 0u, timeout_ns, &abort_flag, status, kDevTimeoutTest);
  }
}

// ------------------------------------------------------------------ launches
static int grid_for(int64_t work_items, int threads) {
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  int64_t g = (work_items + threads - 1) / threads;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

cudaError_t launch_amax(const void* x, bool bf16, int64_t n, uint32_t* amax_bits,
                        cudaStream_t stream) {
  const int grid = grid_for(n / 16 + 1, 256);
  if (bf16) amax_kernel<true><<<grid, 256, 0, stream>>>(x, n, amax_bits);
  else amax_kernel<false><<<grid, 256, 0, stream>>>(x, n, amax_bits);
  return cudaGetLastError();
}

cudaError_t launch_quantize_nvfp4(const void* x, bool bf16, int64_t rows, int64_t k, int layout,
                                  uint8_t* q, uint8_t* sf, float* ts, const uint32_t* amax_bits,
                                  cudaStream_t stream) {
  const int64_t nblocks = (rows * k + 15) / 16;
  const int grid = grid_for(nblocks, 256);
  if (bf16)
    nvfp4_quantize_kernel<true><<<grid, 256, 0, stream>>>(x, rows, k, layout, q, sf, ts, amax_bits);
  else
    nvfp4_quantize_kernel<false><<<grid, 256, 0, stream>>>(x, rows, k, layout, q, sf, ts,
                                                           amax_bits);
  return cudaGetLastError();
}

cudaError_t launch_quantize_mxfp8(const void* x, bool bf16, int64_t rows, int64_t k, int layout,
                                  uint8_t* q, uint8_t* sf, cudaStream_t stream) {
  const int grid = grid_for(rows * (k / 32), 256);
  if (bf16) mxfp8_quantize_kernel<true><<<grid, 256, 0, stream>>>(x, rows, k, layout, q, sf);
  else mxfp8_quantize_kernel<false><<<grid, 256, 0, stream>>>(x, rows, k, layout, q, sf);
  return cudaGetLastError();
}

cudaError_t launch_quantize_mxfp4(const void* x, bool bf16, int64_t rows, int64_t k, int layout,
                                  uint8_t* q, uint8_t* sf, cudaStream_t stream) {
  const int grid = grid_for(rows * (k / 32), 256);
  if (bf16) mxfp4_quantize_kernel<true><<<grid, 256, 0, stream>>>(x, rows, k, layout, q, sf);
  else mxfp4_quantize_kernel<false><<<grid, 256, 0, stream>>>(x, rows, k, layout, q, sf);
  return cudaGetLastError();
}

cudaError_t launch_repack_nvfp4(const uint8_t* sq, const uint8_t* ssf, int src_layout,
                                uint8_t* dq, uint8_t* dsf, int dst_layout, int64_t rows,
                                int64_t k, cudaStream_t stream) {
  const int grid = grid_for(rows * (k / 16), 256);
  nvfp4_repack_kernel<<<grid, 256, 0, stream>>>(sq, ssf, src_layout, dq, dsf, dst_layout, rows,
                                                k);
  return cudaGetLastError();
}

// Exhaustive check of the hardware e2m1 conversion against e2m1_encode (the
// bit-exact restatement of encode_e2m1_rn, e2m1_encode.cuh:18-44) over all
// 2^32 fp32 bit patterns, each converted in both nibble positions.  out[0]:
// mismatches on non-NaN inputs, out[1]: on NaN inputs, out[2]: the largest
// mismatching non-NaN bit pattern + 1 (0 if none).
__global__ void __launch_bounds__(256) e2m1_cvt_selftest_kernel(unsigned long long* out) {
  unsigned long long bad = 0, bad_nan = 0, last = 0;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t u = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
       u < (1ull << 32); u += stride) {
    const float f = __uint_as_float(static_cast<uint32_t>(u));
    const uint32_t want = e2m1_encode(f);
    const uint32_t a = e2m1x2_cvt(f, 0.0f) >> 4;
    const uint32_t b = e2m1x2_cvt(0.0f, f) & 0xfu;
    if (a != want || b != want) {
      if (f != f) {
        ++bad_nan;
      } else {
        ++bad;
        last = u + 1;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    bad += __shfl_xor_sync(0xffffffffu, bad, o);
    bad_nan += __shfl_xor_sync(0xffffffffu, bad_nan, o);
    const unsigned long long l = __shfl_xor_sync(0xffffffffu, last, o);
    last = l > last ? l : last;
  }
  if ((threadIdx.x & 31) == 0) {
    if (bad) atomicAdd(&out[0], bad);
    if (bad_nan) atomicAdd(&out[1], bad_nan);
    if (last) atomicMax(&out[2], last);
  }
}

cudaError_t launch_e2m1_cvt_selftest(unsigned long long* out, cudaStream_t stream) {
  if (cudaMemsetAsync(out, 0, 3 * sizeof(unsigned long long), stream) != cudaSuccess)
    return cudaGetLastError();
  e2m1_cvt_selftest_kernel<<<num_sms() * 8, 256, 0, stream>>>(out);
  return cudaGetLastError();
}

cudaError_t launch_wait_timeout_selftest(uint64_t timeout_ns, uint32_t* status,
                                         cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(timeout_ns, status);
  return cudaGetLastError();
}

}  // namespace qg
