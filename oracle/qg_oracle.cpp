// qg_oracle.cpp -- CPU restatement of the reference's block-scaled GEMM path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
// library in cuda_optimazation_b200/.  Only tests/, __graft_entry__.smoke() and
// bench.py's cpu_baseline / --impl reference legs may load it.  The product
// never links, imports or calls anything built from here.
//
// Every function restates one reference routine (paths are relative to the
// hibouwu/CUDA_optimazation project root):
//   O1  make_nvfp4_reference       GEMMsm110/include/requant/nvfp4_reference.cuh:76-112
//       encode_e2m1_rn             GEMMsm110/include/requant/e2m1_encode.cuh:18-44
//       pack_e2m1x2                GEMMsm110/include/requant/pack_fp4.cuh:11-15
//       decode_positive_e4m3       GEMMsm110/include/requant/nvfp4_reference.cuh:36-48
//       encode_positive_e4m3_round_up  nvfp4_reference.cuh:57-64
//       make_nvfp4_tensor_scale    nvfp4_reference.cuh:66-74
//   O2  block_scaled_reference_mnk cutlass-gemm-cpp-guide/include/guide/block_scale_reference.hpp:10-37
//   L1  sm1xx_scale_offset         cutlass-gemm-cpp-guide/include/guide/scale_layout.hpp:11-26
//       sm1xx_scale_storage_size   scale_layout.hpp:28-34
//   input generators               GEMMsm110/tests/requant_epilogue_benchmark.cu:135-165
//
// MXFP8 has no quantizer in the reference.  qgo_quantize_mxfp8 restates the
// OCP Microscaling Formats (MX) v1.0 rule (shared exponent
// floor(log2(amax)) - emax_elem, emax_elem = 8 for E4M3, stored as E8M0 with
// bias 127, elements RN-satfinite E4M3 of x / 2^e).  Parity for that
// quantizer is therefore unpinned; the MXFP8 GEMM is pinned through O2.
// qgo_mxfp4_quantize restates the same rule for E2M1 elements (emax_elem = 2),
// also unpinned; the MXFP4 GEMM is pinned through O2 with SV = 32.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <random>
#include <thread>
#include <vector>

namespace {

constexpr int kNvfp4Block = 16;
constexpr float kE2M1Max = 6.0f;
constexpr float kE4M3Max = 448.0f;

// e2m1 nibble from fp32 (RNE through bit thresholds, sign kept on zero,
// NaN -> +0, saturate at 6): e2m1_encode.cuh:18-44.
uint8_t encode_e2m1(float v) {
  uint32_t raw;
  std::memcpy(&raw, &v, 4);
  const uint32_t mag = raw & 0x7fffffffu;
  if (mag > 0x7f800000u) return 0u;
  // Each threshold is the lowest fp32 magnitude that encodes to the next
  // e2m1 code; ties at 0.25/1.25/2.5/5.0 go down (even code), ties at
  // 0.75/1.75/3.5 go up (even code).
  static const uint32_t kThresholds[7] = {0x3e800001u, 0x3f400000u, 0x3fa00001u,
                                          0x3fe00000u, 0x40200001u, 0x40600000u,
                                          0x40a00001u};
  uint8_t code = 0;
  for (uint32_t t : kThresholds) code += (mag >= t) ? 1 : 0;
  return static_cast<uint8_t>(((raw >> 28) & 0x8u) | code);
}

float decode_e2m1(uint8_t bits) {
  static const float kMag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float m = kMag[bits & 7u];
  return (bits & 8u) ? -m : m;
}

// nvfp4_reference.cuh:36-48
float decode_e4m3_positive(uint8_t bits) {
  const int e = (bits >> 3) & 0xf;
  const int m = bits & 7;
  if (e == 0) return std::ldexp(static_cast<float>(m), -9);
  if (e == 0xf && m == 7) return std::numeric_limits<float>::quiet_NaN();
  return std::ldexp(1.0f + static_cast<float>(m) / 8.0f, e - 7);
}

// nvfp4_reference.cuh:57-64: the first code 1..0x7e whose value is >= v,
// else the largest finite code.
uint8_t encode_e4m3_round_up(float v) {
  if (!(v > 0.0f)) return 0u;
  for (int c = 1; c <= 0x7e; ++c)
    if (decode_e4m3_positive(static_cast<uint8_t>(c)) >= v) return static_cast<uint8_t>(c);
  return 0x7eu;
}

// Signed e4m3 (bias 7, max 448, no inf) decode for the MXFP8 element path.
float decode_e4m3(uint8_t bits) {
  const float m = decode_e4m3_positive(bits & 0x7fu);
  return (bits & 0x80u) ? -m : m;
}

// Round-to-nearest-even, saturate-to-finite fp32 -> e4m3, written from the
// format definition: enumerate the 127 finite non-negative codes and pick the
// nearest, ties to the even code.  NaN -> 0x7f (e4m3 NaN).
uint8_t encode_e4m3_rn_satfinite(float v) {
  if (std::isnan(v)) return 0x7fu;
  const uint8_t sign = std::signbit(v) ? 0x80u : 0u;
  const float a = std::fabs(v);
  if (a >= kE4M3Max) return sign | 0x7eu;
  // Binary search over monotone codes 0..0x7e.
  int lo = 0, hi = 0x7e;
  while (hi - lo > 1) {
    const int mid = (lo + hi) / 2;
    if (decode_e4m3_positive(static_cast<uint8_t>(mid)) <= a) lo = mid; else hi = mid;
  }
  const double dl = a - static_cast<double>(decode_e4m3_positive(static_cast<uint8_t>(lo)));
  const double dh = static_cast<double>(decode_e4m3_positive(static_cast<uint8_t>(hi))) - a;
  int c;
  if (dl < dh) c = lo;
  else if (dh < dl) c = hi;
  else c = (lo % 2 == 0) ? lo : hi;
  return sign | static_cast<uint8_t>(c);
}

float decode_ue8m0(uint8_t bits) {
  if (bits == 0xffu) return std::numeric_limits<float>::quiet_NaN();
  return std::ldexp(1.0f, static_cast<int>(bits) - 127);
}

}  // namespace

extern "C" {

// ----------------------------------------------------------------- codecs
uint8_t qgo_encode_e2m1(float v) { return encode_e2m1(v); }
float qgo_decode_e2m1(uint8_t b) { return decode_e2m1(b); }
float qgo_decode_e4m3_positive(uint8_t b) { return decode_e4m3_positive(b); }
uint8_t qgo_encode_e4m3_round_up(float v) { return encode_e4m3_round_up(v); }
uint8_t qgo_encode_e4m3_rn(float v) { return encode_e4m3_rn_satfinite(v); }
float qgo_decode_e4m3(uint8_t b) { return decode_e4m3(b); }
float qgo_decode_ue8m0(uint8_t b) { return decode_ue8m0(b); }
// pack_fp4.cuh:11-15: the first logical value goes to the HIGH nibble.
uint8_t qgo_pack_e2m1x2(uint8_t v0, uint8_t v1) {
  return static_cast<uint8_t>(((v0 & 0xfu) << 4) | (v1 & 0xfu));
}

// ----------------------------------------------------------------- layout
// L1, scale_layout.hpp:11-26.  order 0 = the reference's closed form
// (scale-column block outer: block = block_sf * blocks_mn + block_mn);
// order 1 = K-block contiguous (block = block_mn * blocks_sf + block_sf), the
// order CuTe's tile_to_shape(SfAtom, (MN,K), Step<_2,_1>) produces.  Both
// orders agree whenever blocks_mn == 1 or blocks_sf == 1.
int64_t qgo_scale_offset(int64_t mn, int64_t k_element, int64_t mn_extent, int64_t k_extent,
                         int sv, int order) {
  if (mn < 0 || mn >= mn_extent || k_element < 0 || k_element >= k_extent) return -1;
  const int64_t sf = k_element / sv;
  const int64_t blocks_mn = (mn_extent + 127) / 128;
  const int64_t sf_extent = (k_extent + sv - 1) / sv;
  const int64_t blocks_sf = (sf_extent + 3) / 4;
  const int64_t bmn = mn / 128, bsf = sf / 4;
  const int64_t within = mn % 128;
  const int64_t block = order == 0 ? bsf * blocks_mn + bmn : bmn * blocks_sf + bsf;
  return block * 512 + (within % 32) * 16 + (within / 32) * 4 + sf % 4;
}

int64_t qgo_scale_storage_size(int64_t mn_extent, int64_t k_extent, int sv) {
  const int64_t blocks_mn = (mn_extent + 127) / 128;
  const int64_t sf_extent = (k_extent + sv - 1) / sv;
  return blocks_mn * ((sf_extent + 3) / 4) * 512;
}

// ----------------------------------------------------------------- O1
// make_nvfp4_reference over a flat tensor of n elements: nvfp4_reference.cuh:76-112.
// q gets ceil(n_pad/2) bytes (high nibble first), sf gets n_pad/16 bytes
// (linear order), *ts the tensor scale.
void qgo_nvfp4_blocks_with_ts(const float* x, int64_t n, float tscale, uint8_t* q, uint8_t* sf);

void qgo_nvfp4_reference(const float* x, int64_t n, uint8_t* q, uint8_t* sf, float* ts) {
  float amax = 0.0f;
  for (int64_t i = 0; i < n; ++i) amax = std::max(amax, std::fabs(x[i]));
  const float tscale = amax > 0.0f ? amax / (kE4M3Max * kE2M1Max) : 1.0f;
  *ts = tscale;
  qgo_nvfp4_blocks_with_ts(x, n, tscale, q, sf);
}

// The block loop of O1 (nvfp4_reference.cuh:84-111) under a given tensor
// scale: what the tc6 epilogue computes from the inverse tensor scale it is
// handed (tc6_nvfp4.cuh:460-503, Tc6Runner argument at main.cu:2388-2390).
void qgo_nvfp4_blocks_with_ts(const float* x, int64_t n, float tscale, uint8_t* q, uint8_t* sf) {
  const float inv_ts = 1.0f / tscale;
  const int64_t blocks = (n + kNvfp4Block - 1) / kNvfp4Block;
  for (int64_t b = 0; b < blocks; ++b) {
    float vals[kNvfp4Block];
    float namax = 0.0f;
    for (int i = 0; i < kNvfp4Block; ++i) {
      const int64_t idx = b * kNvfp4Block + i;
      vals[i] = idx < n ? x[idx] : 0.0f;
      namax = std::max(namax, std::fabs(vals[i] * inv_ts));
    }
    const uint8_t s = encode_e4m3_round_up(namax / kE2M1Max);
    sf[b] = s;
    const float bs = decode_e4m3_positive(s);
    const float mult = bs > 0.0f ? inv_ts / bs : 0.0f;
    for (int i = 0; i < kNvfp4Block; i += 2) {
      q[(b * kNvfp4Block + i) / 2] =
          qgo_pack_e2m1x2(encode_e2m1(vals[i] * mult), encode_e2m1(vals[i + 1] * mult));
    }
  }
}

// O1 re-expressed for a rows x k matrix (k % 16 == 0) straight into the MMA
// layout: low nibble first, scales at L1 offsets of the given order, padded
// scale slots zero.  Bytes equal a layout conversion of qgo_nvfp4_reference.
void qgo_nvfp4_quantize_mma(const float* x, int64_t rows, int64_t k, int order, uint8_t* q,
                            uint8_t* sf, float* ts) {
  const int64_t n = rows * k;
  std::vector<uint8_t> rq((n + 1) / 2), rsf(n / kNvfp4Block);
  qgo_nvfp4_reference(x, n, rq.data(), rsf.data(), ts);
  for (int64_t i = 0; i < n / 2; ++i) q[i] = static_cast<uint8_t>((rq[i] >> 4) | (rq[i] << 4));
  std::memset(sf, 0, static_cast<size_t>(qgo_scale_storage_size(rows, k, kNvfp4Block)));
  const int64_t sfk = k / kNvfp4Block;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t s = 0; s < sfk; ++s)
      sf[qgo_scale_offset(r, s * kNvfp4Block, rows, k, kNvfp4Block, order)] = rsf[r * sfk + s];
}

// MXFP8 (OCP MX v1.0) for rows x k (k % 32 == 0): q row-major e4m3 bytes,
// scales at L1 offsets (SV = 32) when order >= 0, else linear [rows][k/32].
void qgo_mxfp8_quantize(const float* x, int64_t rows, int64_t k, int order, uint8_t* q,
                        uint8_t* sf) {
  const int sv = 32;
  const int64_t sfk = k / sv;
  if (order >= 0) std::memset(sf, 0, static_cast<size_t>(qgo_scale_storage_size(rows, k, sv)));
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t s = 0; s < sfk; ++s) {
      const float* blk = x + r * k + s * sv;
      float amax = 0.0f;
      for (int i = 0; i < sv; ++i) amax = std::max(amax, std::fabs(blk[i]));
      int e = -127;
      if (amax > 0.0f) {
        int ex;
        std::frexp(amax, &ex);  // amax = f * 2^ex, f in [0.5, 1)
        e = (ex - 1) - 8;        // floor(log2(amax)) - emax(e4m3)
        e = std::max(-127, std::min(127, e));
      }
      const uint8_t code = static_cast<uint8_t>(e + 127);
      if (order >= 0) sf[qgo_scale_offset(r, s * sv, rows, k, sv, order)] = code;
      else sf[r * sfk + s] = code;
      for (int i = 0; i < sv; ++i)
        q[r * k + s * sv + i] = encode_e4m3_rn_satfinite(std::ldexp(blk[i], -e));
    }
  }
}

// ----------------------------------------------------------------- O2
// block_scaled_reference_mnk (block_scale_reference.hpp:10-37) over logical
// fp32 operands, double accumulation, cast to float.  Rows [row_begin,
// row_end) only, spread over `threads` host threads; d holds those rows.
void qgo_block_scaled_gemm(const float* a_mk, const float* b_nk, const float* sfa,
                           const float* sfb, int64_t m, int64_t n, int64_t k, int sv,
                           int64_t row_begin, int64_t row_end, int threads, float* d) {
  (void)m;
  const int64_t sfk = (k + sv - 1) / sv;
  auto work = [&](int64_t r0, int64_t r1) {
    for (int64_t row = r0; row < r1; ++row)
      for (int64_t col = 0; col < n; ++col) {
        double sum = 0.0;
        for (int64_t kk = 0; kk < k; ++kk) {
          const int64_t s = kk / sv;
          const double av = a_mk[row * k + kk], bv = b_nk[col * k + kk];
          const double as = sfa[row * sfk + s], bs = sfb[col * sfk + s];
          sum += (av * as) * (bv * bs);
        }
        d[(row - row_begin) * n + col] = static_cast<float>(sum);
      }
  };
  if (threads <= 1) { work(row_begin, row_end); return; }
  std::vector<std::thread> pool;
  const int64_t total = row_end - row_begin;
  for (int t = 0; t < threads; ++t) {
    const int64_t r0 = row_begin + total * t / threads, r1 = row_begin + total * (t + 1) / threads;
    if (r0 < r1) pool.emplace_back(work, r0, r1);
  }
  for (auto& th : pool) th.join();
}

// Decode MMA-layout NVFP4 operands (low nibble first, L1 scales) into the
// logical fp32 tensors O2 consumes: value [rows][k] and scale [rows][k/16].
void qgo_nvfp4_decode_mma(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t k, int order,
                          float* vals, float* scales) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < k; ++c) {
      const uint8_t byte = q[(r * k + c) / 2];
      vals[r * k + c] = decode_e2m1((c & 1) ? (byte >> 4) : (byte & 0xf));
    }
    for (int64_t s = 0; s < k / 16; ++s)
      scales[r * (k / 16) + s] =
          decode_e4m3_positive(sf[qgo_scale_offset(r, s * 16, rows, k, 16, order)]);
  }
}

// Decode MXFP8 operands (e4m3 bytes, L1 scales with SV 32).
// MXFP4 (OCP MX v1.0 with E2M1 elements; no reference quantizer, parity
// unpinned) for rows x k (k % 32 == 0): shared exponent floor(log2(amax)) - 2
// (emax of E2M1), clamped to [-127, 127], all-zero block -> code 0; elements
// encode_e2m1 (RNE, saturating, NaN -> 0) of x * 2^-e.  order < 0: the
// first element of a pair in the high nibble (pack_fp4.cuh:11-15), scales
// [rows][k/32]; order >= 0: low nibble first, scales at the L1 offsets.
void qgo_mxfp4_quantize(const float* x, int64_t rows, int64_t k, int order, uint8_t* q,
                        uint8_t* sf) {
  const int sv = 32;
  const int64_t sfk = k / sv;
  if (order >= 0) std::memset(sf, 0, static_cast<size_t>(qgo_scale_storage_size(rows, k, sv)));
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t s = 0; s < sfk; ++s) {
      const float* blk = x + r * k + s * sv;
      float amax = 0.0f;
      for (int i = 0; i < sv; ++i) amax = std::max(amax, std::fabs(blk[i]));
      int e = -127;
      if (amax > 0.0f) {
        int ex;
        std::frexp(amax, &ex);  // amax = f * 2^ex, f in [0.5, 1)
        e = std::max(-127, std::min(127, (ex - 1) - 2));
      }
      const uint8_t code = static_cast<uint8_t>(e + 127);
      if (order >= 0) sf[qgo_scale_offset(r, s * sv, rows, k, sv, order)] = code;
      else sf[r * sfk + s] = code;
      for (int i = 0; i < sv; i += 2) {
        const uint8_t c0 = encode_e2m1(std::ldexp(blk[i], -e));
        const uint8_t c1 = encode_e2m1(std::ldexp(blk[i + 1], -e));
        q[(r * k + s * sv + i) / 2] =
            order < 0 ? qgo_pack_e2m1x2(c0, c1) : static_cast<uint8_t>(c0 | (c1 << 4));
      }
    }
  }
}

void qgo_mxfp4_decode(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t k, int order,
                      float* vals, float* scales) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < k; ++c) {
      const uint8_t b = q[(r * k + c) / 2];
      const bool high = (order < 0) == ((c & 1) == 0);
      vals[r * k + c] = decode_e2m1(high ? (b >> 4) : (b & 15));
    }
    for (int64_t s = 0; s < k / 32; ++s)
      scales[r * (k / 32) + s] = decode_ue8m0(
          order >= 0 ? sf[qgo_scale_offset(r, s * 32, rows, k, 32, order)] : sf[r * (k / 32) + s]);
  }
}

void qgo_mxfp8_decode(const uint8_t* q, const uint8_t* sf, int64_t rows, int64_t k, int order,
                      float* vals, float* scales) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < k; ++c) vals[r * k + c] = decode_e4m3(q[r * k + c]);
    for (int64_t s = 0; s < k / 32; ++s)
      scales[r * (k / 32) + s] = decode_ue8m0(
          order >= 0 ? sf[qgo_scale_offset(r, s * 32, rows, k, 32, order)] : sf[r * (k / 32) + s]);
  }
}

// ----------------------------------------------------------------- inputs
// Seeded N(mean, std) fill: std::mt19937_64 + std::normal_distribution<float>.
void qgo_fill_normal(float* out, int64_t n, uint64_t seed, float mean, float stddev) {
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> dist(mean, stddev);
  for (int64_t i = 0; i < n; ++i) out[i] = dist(rng);
}

// The six distributions of requant_epilogue_benchmark.cu:135-165, with the
// same engine (std::mt19937, 32-bit) and draw order.
// dist: 0 uniform, 1 normal, 2 laplace, 3 outlier, 4 lognormal, 5 constant.
void qgo_fill_requant_dist(float* out, int64_t n, uint32_t seed, int dist) {
  std::mt19937 rng(seed);
  std::uniform_real_distribution<float> uniform(-1.0f, 1.0f);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  std::exponential_distribution<float> exponential(1.0f);
  std::lognormal_distribution<float> lognormal(0.0f, 1.25f);
  std::bernoulli_distribution sign(0.5);
  for (int64_t i = 0; i < n; ++i) {
    float v;
    switch (dist) {
      case 0: v = uniform(rng); break;
      case 1: v = normal(rng); break;
      case 2: v = exponential(rng) * (sign(rng) ? 1.0f : -1.0f); break;
      case 3: v = normal(rng); if (i % 257 == 0) v *= 128.0f; break;
      case 4: v = lognormal(rng) * (sign(rng) ? 1.0f : -1.0f); break;
      default: v = 0.75f; break;
    }
    out[i] = v;
  }
}

}  // extern "C"
