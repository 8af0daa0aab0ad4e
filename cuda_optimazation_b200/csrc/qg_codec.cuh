// qg_codec.cuh -- NVFP4 element / scale codecs and vector loads shared by the
// activation quantizers (quantize.cu, gemm_skinny.cu).  Rounding follows
// make_nvfp4_reference (GEMMsm110/include/requant/nvfp4_reference.cuh:76-112).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace qg {

// ------------------------------------------------------------------ codecs
// fp32 -> e2m1 nibble, round to nearest even, sign kept on zero, NaN -> +0,
// saturating at 6.  The seven thresholds are the fp32 bit patterns of the
// rounding boundaries of the e2m1 grid {0, .5, 1, 1.5, 2, 3, 4, 6}: a tie
// that must round to the even lower code starts one ulp above the midpoint.
__device__ __forceinline__ uint32_t e2m1_encode(float v) {
  const uint32_t raw = __float_as_uint(v);
  const uint32_t mag = raw & 0x7fffffffu;
  if (mag > 0x7f800000u) return 0u;
  const uint32_t code = (mag >= 0x3e800001u) + (mag >= 0x3f400000u) + (mag >= 0x3fa00001u) +
                        (mag >= 0x3fe00000u) + (mag >= 0x40200001u) + (mag >= 0x40600000u) +
                        (mag >= 0x40a00001u);
  return ((raw >> 28) & 0x8u) | code;
}

// Smallest positive finite e4m3 code whose value is >= v (0 for v <= 0,
// 0x7e = 448 above the range).  Normal range: truncate the fp32 mantissa to
// 3 bits and bump by one code when any dropped bit is set; subnormal range
// (v < 2^-6): ceil(v * 2^9) subnormal steps.
__device__ __forceinline__ uint32_t e4m3_round_up(float v) {
  if (!(v > 0.0f)) return 0u;
  if (v >= 448.0f) return 0x7eu;
  if (v < 0.015625f) return static_cast<uint32_t>(ceilf(v * 512.0f));
  const uint32_t b = __float_as_uint(v);
  const uint32_t e = ((b >> 23) & 0xffu) - 127u + 7u;
  uint32_t code = (e << 3) | ((b >> 20) & 7u);
  if (b & 0xfffffu) code += 1u;
  return code;
}

__device__ __forceinline__ float e4m3_decode_positive(uint32_t c) {
  const uint32_t e = (c >> 3) & 0xfu, m = c & 7u;
  if (e == 0u) return static_cast<float>(m) * 0.001953125f;  // m * 2^-9
  return __uint_as_float(((e + 120u) << 23) | (m << 20));
}

// Byte offset of scale (row, scale column) in an MMA scale layout.
__device__ __forceinline__ int64_t mma_scale_offset(int64_t row, int64_t sfc, int64_t row_blocks,
                                                    int64_t sf_blocks, int layout) {
  const int64_t br = row >> 7, bs = sfc >> 2, w = row & 127;
  const int64_t chunk = (layout == 1) ? bs * row_blocks + br : br * sf_blocks + bs;
  return chunk * 512 + (w & 31) * 16 + (w >> 5) * 4 + (sfc & 3);
}

template <bool kBf16>
__device__ __forceinline__ void load16(const void* x, int64_t elem, float (&v)[16]) {
  if (kBf16) {
    const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + elem);
    const uint4 a = __ldg(p), b = __ldg(p + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + elem);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = __ldg(p + i);
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
  }
}

template <bool kBf16>
__device__ __forceinline__ float load1(const void* x, int64_t i) {
  if (kBf16) {
    const uint16_t h = reinterpret_cast<const uint16_t*>(x)[i];
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
  }
  return reinterpret_cast<const float*>(x)[i];
}

// Raw 16-element block (bf16: 32 bytes, fp32: 64 bytes), so several blocks'
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

// One 16-element NVFP4 block in the MMA order (low nibble first): returns the
// ue4m3 scale code, packs the 16 e2m1 codes into lo/hi.
__device__ __forceinline__ uint32_t nvfp4_encode_block(const float (&v)[16], float inv_ts,
                                                       uint32_t& lo, uint32_t& hi) {
  float bmax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bmax = fmaxf(bmax, fabsf(v[i]));
  const float namax = __fmul_rn(bmax, inv_ts);  // == max|x * inv_ts| (RN is monotonic)
  const uint32_t sbits = e4m3_round_up(__fdiv_rn(namax, 6.0f));
  const float bs = e4m3_decode_positive(sbits);
  const float mult = bs > 0.0f ? __fdiv_rn(inv_ts, bs) : 0.0f;
  lo = 0;
  hi = 0;
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const uint32_t byte =
        e2m1_encode(__fmul_rn(v[i], mult)) | (e2m1_encode(__fmul_rn(v[i + 1], mult)) << 4);
    if (i < 8) lo |= byte << (4 * i);
    else hi |= byte << (4 * (i - 8));
  }
  return sbits;
}

// Two fp32 values -> one byte of e2m1 codes with the hardware conversion
// (round to nearest even, saturating at +-6): `hi` lands in bits 7..4, `lo` in
// bits 3..0.  For every non-NaN fp32 input the code equals e2m1_encode's
// (checked over all 2^32 bit patterns on the GPU by
// qg_selftest_e2m1_cvt); NaN inputs are mapped to +0 by the caller, as
// e2m1_encode does.
__device__ __forceinline__ uint32_t e2m1x2_cvt(float hi, float lo) {
  uint32_t out;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out;
}

// nvfp4_encode_block with the hardware e2m1 conversion (the requantising GEMM
// epilogue's form): same scale and same codes, low nibble first; `bmax` is
// the block's max |v| (NaN-free, as fmaxf drops NaN operands).
__device__ __forceinline__ uint32_t nvfp4_encode_block_cvt(const float (&v)[16], float bmax,
                                                           float inv_ts, uint32_t& lo,
                                                           uint32_t& hi) {
  const float namax = __fmul_rn(bmax, inv_ts);
  const uint32_t sbits = e4m3_round_up(__fdiv_rn(namax, 6.0f));
  const float bs = e4m3_decode_positive(sbits);
  const float mult = bs > 0.0f ? __fdiv_rn(inv_ts, bs) : 0.0f;
  lo = 0;
  hi = 0;
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    float x0 = __fmul_rn(v[i], mult), x1 = __fmul_rn(v[i + 1], mult);
    x0 = x0 == x0 ? x0 : 0.0f;  // NaN -> +0
    x1 = x1 == x1 ? x1 : 0.0f;
    const uint32_t byte = e2m1x2_cvt(x1, x0);
    if (i < 8) lo |= byte << (4 * i);
    else hi |= byte << (4 * (i - 8));
  }
  return sbits;
}

}  // namespace qg
