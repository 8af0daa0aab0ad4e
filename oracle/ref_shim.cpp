// ref_shim.cpp -- C entry points over the reference's OWN host oracles.
//
// TEST INFRASTRUCTURE ONLY (see qg_oracle.cpp).  This file holds no algorithm:
// it includes the reference headers where they lie (include path set by
// oracle/Makefile, REF=<reference checkout>) and wraps them in extern "C" so
// the tests can pin qg_oracle.cpp against the reference itself, and so
// bench.py's reference arm can time the reference's own CPU path.
//   make_nvfp4_reference       GEMMsm110/include/requant/nvfp4_reference.cuh:76-112
//   encode_e2m1_rn             GEMMsm110/include/requant/e2m1_encode.cuh:18-44
//   block_scaled_reference_mnk cutlass-gemm-cpp-guide/include/guide/block_scale_reference.hpp:10-37
//   sm1xx_scale_offset         cutlass-gemm-cpp-guide/include/guide/scale_layout.hpp:11-26
#include "requant/nvfp4_reference.cuh"
#include "guide/block_scale_reference.hpp"
#include "guide/scale_layout.hpp"

#include <cstring>
#include <thread>
#include <vector>

extern "C" {

uint8_t qgr_encode_e2m1(float v) { return gemm_sm110::requant::encode_e2m1_rn(v); }
uint8_t qgr_encode_e4m3_round_up(float v) {
  return gemm_sm110::requant::encode_positive_e4m3_round_up(v);
}
float qgr_decode_e4m3_positive(uint8_t b) { return gemm_sm110::requant::decode_positive_e4m3(b); }

// Flat-tensor NVFP4 quantisation by the reference.  q: ceil(pad/2) bytes,
// sf: pad/16 bytes.
void qgr_nvfp4_reference(const float* x, int64_t n, uint8_t* q, uint8_t* sf, float* ts) {
  std::vector<float> in(x, x + n);
  auto r = gemm_sm110::requant::make_nvfp4_reference(in);
  std::memcpy(q, r.quantized.data(), r.quantized.size());
  std::memcpy(sf, r.block_scales.data(), r.block_scales.size());
  *ts = r.tensor_scale;
}

int64_t qgr_scale_offset(int mn, int k_element, int mn_extent, int k_extent, int sv) {
  return static_cast<int64_t>(guide::sm1xx_scale_offset(mn, k_element, mn_extent, k_extent, sv));
}
int64_t qgr_scale_storage_size(int mn_extent, int k_extent, int sv) {
  return static_cast<int64_t>(guide::sm1xx_scale_storage_size(mn_extent, k_extent, sv));
}

// The reference O2 over rows [row_begin,row_end) of A; the reference function
// is single-threaded, so `threads` workers each call it on a row slice.
void qgr_block_scaled_gemm(const float* a_mk, const float* b_nk, const float* sfa,
                           const float* sfb, int m, int n, int k, int sv, int row_begin,
                           int row_end, int threads, float* d) {
  (void)m;
  const int sfk = (k + sv - 1) / sv;
  const std::vector<float> b(b_nk, b_nk + static_cast<size_t>(n) * k);
  const std::vector<float> bs(sfb, sfb + static_cast<size_t>(n) * sfk);
  auto work = [&](int r0, int r1) {
    const int rows = r1 - r0;
    std::vector<float> a(a_mk + static_cast<size_t>(r0) * k, a_mk + static_cast<size_t>(r1) * k);
    std::vector<float> as(sfa + static_cast<size_t>(r0) * sfk, sfa + static_cast<size_t>(r1) * sfk);
    auto out = guide::block_scaled_reference_mnk(a, b, as, bs, rows, n, k, sv);
    std::memcpy(d + static_cast<size_t>(r0 - row_begin) * n, out.data(), out.size() * 4);
  };
  if (threads < 1) threads = 1;
  std::vector<std::thread> pool;
  const int total = row_end - row_begin;
  for (int t = 0; t < threads; ++t) {
    const int r0 = row_begin + total * t / threads, r1 = row_begin + total * (t + 1) / threads;
    if (r0 < r1) pool.emplace_back(work, r0, r1);
  }
  for (auto& th : pool) th.join();
}

}  // extern "C"
