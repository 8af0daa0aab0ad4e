// capi.cu -- host side of the C ABI declared in include/qgemm.h.
//
// Validates shapes / alignment / layouts, encodes the TMA tensor maps
// (cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library needs no link-time libcuda), and launches the kernels.  It never
// allocates device memory and never exits the process.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>

#include "../../include/qgemm.h"
#include "qg_gemm.h"

namespace qg {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QG_ERR_CUDA;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return QG_ERR_CUDA;
  return major == 10 ? QG_OK : QG_ERR_UNSUPPORTED;
}

// Operand values: uint8 [rows][row_bytes], box 128 B x box_rows, SWIZZLE_128B.
bool make_operand_map(CUtensorMap* m, const void* base, int64_t rows, int64_t row_bytes,
                      int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1u, 1u};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Scale chunks: uint32 [scale_blocks][row_blocks][128] with the chunk
// strides of the chosen MMA order; box (128, box_row_blocks, box_chunks).
bool make_scale_map(CUtensorMap* m, const void* base, int64_t mn, int64_t k, int sv, int layout,
                    int box_row_blocks, int box_chunks) {
  const int64_t row_blocks = (mn + 127) / 128;
  const int64_t sf_blocks = ((k + sv - 1) / sv + 3) / 4;
  const cuuint64_t dims[3] = {128u, static_cast<cuuint64_t>(row_blocks),
                              static_cast<cuuint64_t>(sf_blocks)};
  cuuint64_t strides[2];
  if (layout == QG_LAYOUT_MMA) {
    strides[0] = 512u;
    strides[1] = static_cast<cuuint64_t>(row_blocks) * 512u;
  } else {
    strides[0] = static_cast<cuuint64_t>(sf_blocks) * 512u;
    strides[1] = 512u;
  }
  const cuuint32_t box[3] = {128u, static_cast<cuuint32_t>(box_row_blocks),
                             static_cast<cuuint32_t>(box_chunks)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 output [rows][cols] with row stride ldc elements, as 64-column x
// 32-row TMA store boxes with the 128-byte swizzle of the staging buffer.
bool make_output_map(CUtensorMap* map, void* base, int64_t rows, int64_t cols, int64_t ldc) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldc * 2)};
  const cuuint32_t box[2] = {64u, 32u};
  const cuuint32_t estr[2] = {1u, 1u};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint64_t default_timeout_ns() {
  static uint64_t t = [] {
    const char* e = std::getenv("QG_WAIT_TIMEOUT_NS");
    return e ? static_cast<uint64_t>(std::strtoull(e, nullptr, 10)) : 2000000000ull;
  }();
  return t;
}

// GEMM kernel variant: 0 = single CTA with tcgen05.st scale staging,
// 1 = CTA pair with tcgen05.st staging, 2 = single CTA with tcgen05.cp scale
// copies.  Measured on B200 (8192^3 NVFP4 / 4096x14336x4096 MXFP8): the pair
// kernel wins whenever a 256-row tile is filled (NVFP4 8192^3 4.6 vs 3.9 PF/s
// solo; MXFP8 2.34 vs 2.06 PF/s 1-CTA); problems of at most 128 rows use one
// CTA per tile (the pair's 256-row tile would be half empty).  A build with
// -DQG_GEMM_VARIANT=<0|1|2> forces one variant for A/B measurements; the
// shipped library has no runtime switch.
int gemm_variant(bool fp4, int64_t m) {
#ifdef QG_GEMM_VARIANT
  return QG_GEMM_VARIANT;
#endif
  if (m > 128) return 1;
  return fp4 ? 0 : 2;
}

// The bf16 TMA-store epilogue of the pair kernel runs on eight warps; a
// build with -DQG_PAIR_EPI4 selects the older four-warp form (A/B runs).
constexpr bool kPairEpi8 =
#ifdef QG_PAIR_EPI4
    false;
#else
    true;
#endif

// `gather` (fused column-parallel output gather): this GPU computes the
// columns [col0, col0 + n) of a C with row stride ldc and stores them into
// every buffer of c_ranks (nranks of them, peer buffers IPC-mapped); only the
// pair kernel with bf16 output does this.
struct Gather {
  void* const* c_ranks = nullptr;
  int nranks = 0;
  int64_t col0 = 0;
};

// `requant` (q != null): NVFP4 output written by the pair kernel's
// requantising epilogue instead of C (c / c_dtype / ldc unused).
struct Requant {
  uint8_t* q = nullptr;
  uint8_t* sf = nullptr;
  const float* ts = nullptr;
  uint32_t* amax = nullptr;
  int layout = 0;
};

// A GEMM call with everything host-side done: shapes checked, tensor maps
// encoded, kernel variant and grid chosen.  gemm_launch() enqueues it;
// qg_plan keeps one to skip the host work on repeated calls.
struct PreparedGemm {
  GemmParams p;
  int fmt = 1;
  bool fp4 = true, pair = true, out_bf16 = false;
  int variant = 1, out_kind = 0, grid = 0;
  void* memset_ptr = nullptr;  // scale padding to clear before each launch
  size_t memset_bytes = 0;
};

cudaError_t gemm_launch(const PreparedGemm& g, cudaStream_t stream) {
  if (g.memset_bytes) {
    cudaError_t e = cudaMemsetAsync(g.memset_ptr, 0, g.memset_bytes, stream);
    if (e != cudaSuccess) return e;
  }
  if (g.pair) return launch_gemm_pair(g.p, g.fmt, g.out_kind, g.grid, stream);
  return g.variant == 2 ? launch_gemm_blockscaled(g.p, g.fp4, g.out_bf16, g.grid, stream)
                        : launch_gemm_solo(g.p, g.fp4, g.out_bf16, g.grid, stream);
}

// fmt: 0 MXFP8, 1 NVFP4, 2 MXFP4 (pair kernel only).
int gemm_prepare(int fmt, const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                 const void* b_sf, const float* b_ts, void* c, int c_dtype, int64_t m, int64_t n,
                 int64_t k, int64_t ldc, int sf_layout, uint32_t* status, PreparedGemm* out,
                 const Gather& gather = Gather(), const Requant& requant = Requant()) {
  const bool rq = requant.q != nullptr;
  const bool fp4 = fmt != 0;
  if (!a_q || !a_sf || !b_q || !b_sf || (!c && !rq)) return QG_ERR_ARG;
  if (!rq && c_dtype != QG_DTYPE_F32 && c_dtype != QG_DTYPE_BF16) return QG_ERR_DTYPE;
  if (sf_layout != QG_LAYOUT_MMA && sf_layout != QG_LAYOUT_MMA_KMAJOR) return QG_ERR_LAYOUT;
  if (m < 1 || n < 1 || k < 32 || (k % 32) != 0 || ldc < n) return QG_ERR_SHAPE;
  if (m > (1ll << 31) - 1 || n > (1ll << 31) - 1 || k > (1ll << 31) - 1) return QG_ERR_SHAPE;
  if (!aligned16(a_q) || !aligned16(b_q) || !aligned16(a_sf) || !aligned16(b_sf))
    return QG_ERR_ALIGN;
  const int64_t row_bytes = fp4 ? k / 2 : k;
  if (row_bytes % 16 != 0) return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  if (!encode_fn()) return QG_ERR_CUDA;
  const int sv = fmt == 1 ? 16 : 32;
  const int variant = (gather.nranks > 0 || rq || fmt == 2) ? 1 : gemm_variant(fp4, m);
  const bool pair = variant == 1;
  // Tile of one scheduling unit (a CTA pair: 256 x 256; one CTA: 128 x 256)
  // and the rows each CTA's TMA boxes cover.
  const int tm = pair ? pair_tile_m() : gemm_tile_m();
  const int tn = pair ? pair_tile_n() : gemm_tile_n();
  const int box_a = pair ? tm / 2 : tm;
  const int box_b = pair ? tn / 2 : tn;
  const int chunks = pair ? pair_sf_chunks_per_stage(fmt) : gemm_sf_chunks_per_stage(fp4);
  GemmParams& p = out->p;
  std::memset(&p, 0, sizeof(p));
  if (!make_operand_map(&p.tm_a, a_q, m, row_bytes, box_a)) return QG_ERR_CUDA;
  if (!make_operand_map(&p.tm_b, b_q, n, row_bytes, box_b)) return QG_ERR_CUDA;
  if (!make_scale_map(&p.tm_sfa, a_sf, m, k, sv, sf_layout, box_a / 128, chunks)) return QG_ERR_CUDA;
  if (!make_scale_map(&p.tm_sfb, b_sf, n, k, sv, sf_layout, tn / 128, chunks)) return QG_ERR_CUDA;
  const int esize = c_dtype == QG_DTYPE_BF16 ? 2 : 4;
  p.c = c;
  p.ldc = ldc;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.num_m_tiles = static_cast<int>((m + tm - 1) / tm);
  p.num_n_tiles = static_cast<int>((n + tn - 1) / tn);
  p.num_k_blocks = static_cast<int>((row_bytes + gemm_stage_k_bytes() - 1) / gemm_stage_k_bytes());
  p.vec_ok = aligned16(c) && ((ldc * esize) % 16 == 0);
  if (gather.nranks > 0) {
    if (esize != 2 || !p.vec_ok || (gather.col0 % 8) != 0) return QG_ERR_ALIGN;
    for (int r = 0; r < gather.nranks; ++r) {
      if (!gather.c_ranks[r] || !aligned16(gather.c_ranks[r])) return QG_ERR_ALIGN;
      uint16_t* base = static_cast<uint16_t*>(gather.c_ranks[r]) + gather.col0;
      if (!make_output_map(&p.tm_out[r], base, m, n, ldc)) return QG_ERR_CUDA;
    }
    p.n_out = gather.nranks;
  } else if (pair && esize == 2 && p.vec_ok) {
    if (!make_output_map(&p.tm_out[0], c, m, n, ldc)) return QG_ERR_CUDA;
    p.n_out = 1;
  }
  if (rq) {
    // Padded scale slots of the MMA layouts must read as zero scales.
    if (requant.layout != QG_LAYOUT_REF_LINEAR && ((m % 128) != 0 || ((n / 16) % 4) != 0)) {
      out->memset_ptr = requant.sf;
      out->memset_bytes = static_cast<size_t>(qg_scale_bytes(m, n, 16));
    }
    p.vec_ok = 0;
    p.n_out = 0;
    p.rq_q = requant.q;
    p.rq_sf = requant.sf;
    p.rq_ts = requant.ts;
    p.rq_amax = requant.amax;
    p.rq_layout = requant.layout;
    p.rq_row_blocks = static_cast<int>((m + 127) / 128);
    p.rq_sf_blocks = static_cast<int>((n / 16 + 3) / 4);
  }
  p.a_ts = fmt == 1 ? a_ts : nullptr;
  p.b_ts = fmt == 1 ? b_ts : nullptr;
  p.status = status;
  p.timeout_ns = default_timeout_ns();
  const int64_t tiles = static_cast<int64_t>(p.num_m_tiles) * p.num_n_tiles;
  out->fmt = fmt;
  out->fp4 = fp4;
  out->pair = pair;
  out->variant = variant;
  out->out_bf16 = c_dtype == QG_DTYPE_BF16;
  if (pair) {
    // One CTA pair per tile: the pairs that fit run persistently and take
    // the rest of the tiles with cluster launch control (gemm_pair.cu).
    if (2 * tiles > (1ll << 31) - 1) return QG_ERR_SHAPE;
    out->grid = 2 * static_cast<int>(tiles);
    // bf16 through TMA stores: the eight-warp epilogue (kind 3).
    out->out_kind = rq ? 2 : (out->out_bf16 ? (p.n_out > 0 && kPairEpi8 ? 3 : 1) : 0);
  } else {
    out->grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  }
  return QG_OK;
}

int gemm_common(int fmt, const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                const void* b_sf, const float* b_ts, void* c, int c_dtype, int64_t m, int64_t n,
                int64_t k, int64_t ldc, int sf_layout, uint32_t* status, cudaStream_t stream,
                const Gather& gather = Gather(), const Requant& requant = Requant()) {
  PreparedGemm g;
  const int rc = gemm_prepare(fmt, a_q, a_sf, a_ts, b_q, b_sf, b_ts, c, c_dtype, m, n, k, ldc,
                              sf_layout, status, &g, gather, requant);
  if (rc != QG_OK) return rc;
  return gemm_launch(g, stream) == cudaSuccess ? QG_OK : QG_ERR_CUDA;
}

}  // namespace

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

}  // namespace qg

using namespace qg;

struct qg_plan_st {
  qg::PreparedGemm gemm;
  int device = 0;
};

extern "C" {

const char* qg_status_string(int s) {
  switch (s) {
    case QG_OK: return "ok";
    case QG_ERR_SHAPE: return "unsupported shape";
    case QG_ERR_ALIGN: return "misaligned pointer or leading dimension";
    case QG_ERR_LAYOUT: return "layout not accepted here";
    case QG_ERR_DTYPE: return "unknown dtype";
    case QG_ERR_CUDA: return "CUDA error";
    case QG_ERR_TIMEOUT: return "device wait timed out";
    case QG_ERR_ARG: return "bad argument";
    case QG_ERR_UNSUPPORTED: return "device is not sm_100";
    default: return "unknown status";
  }
}

const char* qg_version(void) { return "qgemm-b200 0.1.0 (sm_100a)"; }

int64_t qg_scale_bytes(int64_t mn, int64_t k, int sv) {
  if (mn < 0 || k < 0 || sv <= 0) return -1;
  return ((mn + 127) / 128) * (((k + sv - 1) / sv + 3) / 4) * 512;
}

size_t qg_quantize_workspace_bytes(void) { return 256; }

int qg_quantize_nvfp4(const void* x, int x_dtype, int64_t rows, int64_t k, int layout, void* q,
                      void* sf, float* ts, void* workspace, qg_stream_t stream) {
  if (!x || !q || !sf || !workspace) return QG_ERR_ARG;
  if (x_dtype != QG_DTYPE_F32 && x_dtype != QG_DTYPE_BF16) return QG_ERR_DTYPE;
  if (layout < QG_LAYOUT_REF_LINEAR || layout > QG_LAYOUT_MMA_KMAJOR) return QG_ERR_LAYOUT;
  if (rows < 1 || k < 1) return QG_ERR_SHAPE;
  if (layout != QG_LAYOUT_REF_LINEAR && (k % 16) != 0) return QG_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(q) || !aligned16(workspace)) return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf16 = x_dtype == QG_DTYPE_BF16;
  uint32_t* amax = static_cast<uint32_t*>(workspace);
  if (cudaMemsetAsync(amax, 0, sizeof(uint32_t), s) != cudaSuccess) return QG_ERR_CUDA;
  if (layout != QG_LAYOUT_REF_LINEAR && ((rows % 128) != 0 || ((k / 16) % 4) != 0)) {
    // Padded scale slots must read as zero scales.
    if (cudaMemsetAsync(sf, 0, static_cast<size_t>(qg_scale_bytes(rows, k, 16)), s) != cudaSuccess)
      return QG_ERR_CUDA;
  }
  if (launch_amax(x, bf16, rows * k, amax, s) != cudaSuccess) return QG_ERR_CUDA;
  if (launch_quantize_nvfp4(x, bf16, rows, k, layout, static_cast<uint8_t*>(q),
                            static_cast<uint8_t*>(sf), ts, amax, s) != cudaSuccess)
    return QG_ERR_CUDA;
  return QG_OK;
}

int qg_quantize_mxfp8(const void* x, int x_dtype, int64_t rows, int64_t k, int layout, void* q,
                      void* sf, qg_stream_t stream) {
  if (!x || !q || !sf) return QG_ERR_ARG;
  if (x_dtype != QG_DTYPE_F32 && x_dtype != QG_DTYPE_BF16) return QG_ERR_DTYPE;
  if (layout < QG_LAYOUT_REF_LINEAR || layout > QG_LAYOUT_MMA_KMAJOR) return QG_ERR_LAYOUT;
  if (rows < 1 || k < 32 || (k % 32) != 0) return QG_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(q)) return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (layout != QG_LAYOUT_REF_LINEAR && ((rows % 128) != 0 || ((k / 32) % 4) != 0)) {
    if (cudaMemsetAsync(sf, 0, static_cast<size_t>(qg_scale_bytes(rows, k, 32)), s) != cudaSuccess)
      return QG_ERR_CUDA;
  }
  return launch_quantize_mxfp8(x, x_dtype == QG_DTYPE_BF16, rows, k, layout,
                               static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf),
                               s) == cudaSuccess
             ? QG_OK
             : QG_ERR_CUDA;
}

int qg_repack_nvfp4(const void* src_q, const void* src_sf, int src_layout, void* dst_q,
                    void* dst_sf, int dst_layout, int64_t rows, int64_t k, qg_stream_t stream) {
  if (!src_q || !src_sf || !dst_q || !dst_sf) return QG_ERR_ARG;
  if (src_layout < 0 || src_layout > 2 || dst_layout < 0 || dst_layout > 2) return QG_ERR_LAYOUT;
  if (rows < 1 || k < 16 || (k % 16) != 0) return QG_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(src_q) & 7u) || (reinterpret_cast<uintptr_t>(dst_q) & 7u))
    return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dst_layout != QG_LAYOUT_REF_LINEAR && ((rows % 128) != 0 || ((k / 16) % 4) != 0)) {
    if (cudaMemsetAsync(dst_sf, 0, static_cast<size_t>(qg_scale_bytes(rows, k, 16)), s) !=
        cudaSuccess)
      return QG_ERR_CUDA;
  }
  return launch_repack_nvfp4(static_cast<const uint8_t*>(src_q),
                             static_cast<const uint8_t*>(src_sf), src_layout,
                             static_cast<uint8_t*>(dst_q), static_cast<uint8_t*>(dst_sf),
                             dst_layout, rows, k, s) == cudaSuccess
             ? QG_OK
             : QG_ERR_CUDA;
}

int qg_repack_mx(int elem_bits, const void* src_q, const void* src_sf, int src_layout,
                 void* dst_q, void* dst_sf, int dst_layout, int64_t rows, int64_t k,
                 qg_stream_t stream) {
  if (!src_q || !src_sf || !dst_q || !dst_sf) return QG_ERR_ARG;
  if (elem_bits != 4 && elem_bits != 8) return QG_ERR_DTYPE;
  if (src_layout < 0 || src_layout > 2 || dst_layout < 0 || dst_layout > 2) return QG_ERR_LAYOUT;
  if (rows < 1 || k < 32 || (k % 32) != 0) return QG_ERR_SHAPE;
  if (!aligned16(src_q) || !aligned16(dst_q)) return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dst_layout != QG_LAYOUT_REF_LINEAR && ((rows % 128) != 0 || ((k / 32) % 4) != 0)) {
    if (cudaMemsetAsync(dst_sf, 0, static_cast<size_t>(qg_scale_bytes(rows, k, 32)), s) !=
        cudaSuccess)
      return QG_ERR_CUDA;
  }
  return launch_repack_mx(elem_bits == 4, static_cast<const uint8_t*>(src_q),
                          static_cast<const uint8_t*>(src_sf), src_layout,
                          static_cast<uint8_t*>(dst_q), static_cast<uint8_t*>(dst_sf), dst_layout,
                          rows, k, s) == cudaSuccess
             ? QG_OK
             : QG_ERR_CUDA;
}

int qg_gemm_nvfp4(const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                  const void* b_sf, const float* b_ts, void* c, int c_dtype, int64_t m, int64_t n,
                  int64_t k, int64_t ldc, int sf_layout, uint32_t* status, qg_stream_t stream) {
  return gemm_common(1, a_q, a_sf, a_ts, b_q, b_sf, b_ts, c, c_dtype, m, n, k, ldc, sf_layout,
                     status, reinterpret_cast<cudaStream_t>(stream));
}

int qg_gemm_nvfp4_requant(const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                          const void* b_sf, const float* b_ts, const float* out_ts, void* out_q,
                          void* out_sf, int out_layout, uint32_t* out_amax, int64_t m, int64_t n,
                          int64_t k, int sf_layout, uint32_t* status, qg_stream_t stream) {
  if (!out_q || !out_sf) return QG_ERR_ARG;
  if (out_layout < QG_LAYOUT_REF_LINEAR || out_layout > QG_LAYOUT_MMA_KMAJOR) return QG_ERR_LAYOUT;
  if (n < 16 || (n % 16) != 0) return QG_ERR_SHAPE;
  if (!aligned16(out_q) || (reinterpret_cast<uintptr_t>(out_sf) & 3u) ||
      (out_amax && (reinterpret_cast<uintptr_t>(out_amax) & 3u)))
    return QG_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  Requant r;
  r.q = static_cast<uint8_t*>(out_q);
  r.sf = static_cast<uint8_t*>(out_sf);
  r.ts = out_ts;
  r.amax = out_amax;
  r.layout = out_layout;
  return gemm_common(1, a_q, a_sf, a_ts, b_q, b_sf, b_ts, nullptr, QG_DTYPE_F32, m, n, k, n,
                     sf_layout, status, s, Gather(), r);
}

int qg_plan_create_gemm(qg_plan* plan, int format, const void* a_q, const void* a_sf,
                        const float* a_ts, const void* b_q, const void* b_sf, const float* b_ts,
                        void* c, int c_dtype, int64_t m, int64_t n, int64_t k, int64_t ldc,
                        int sf_layout, uint32_t* status) {
  if (!plan) return QG_ERR_ARG;
  *plan = nullptr;
  if (format < QG_FORMAT_MXFP8 || format > QG_FORMAT_MXFP4) return QG_ERR_DTYPE;
  qg_plan_st* pl = new (std::nothrow) qg_plan_st();
  if (!pl) return QG_ERR_ARG;
  const int rc = gemm_prepare(format, a_q, a_sf, a_ts, b_q, b_sf, b_ts, c, c_dtype, m, n, k, ldc,
                              sf_layout, status, &pl->gemm);
  if (rc != QG_OK || cudaGetDevice(&pl->device) != cudaSuccess) {
    delete pl;
    return rc != QG_OK ? rc : QG_ERR_CUDA;
  }
  *plan = pl;
  return QG_OK;
}

int qg_plan_run(qg_plan plan, qg_stream_t stream) {
  if (!plan) return QG_ERR_ARG;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return QG_ERR_CUDA;
  if (dev != plan->device) return QG_ERR_ARG;
  return gemm_launch(plan->gemm, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
             ? QG_OK
             : QG_ERR_CUDA;
}

int qg_plan_destroy(qg_plan plan) {
  if (!plan) return QG_ERR_ARG;
  delete plan;
  return QG_OK;
}

int qg_gemm_mxfp4(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf, void* c,
                  int c_dtype, int64_t m, int64_t n, int64_t k, int64_t ldc, int sf_layout,
                  uint32_t* status, qg_stream_t stream) {
  return gemm_common(2, a_q, a_sf, nullptr, b_q, b_sf, nullptr, c, c_dtype, m, n, k, ldc,
                     sf_layout, status, reinterpret_cast<cudaStream_t>(stream));
}

int qg_quantize_mxfp4(const void* x, int x_dtype, int64_t rows, int64_t k, int layout, void* q,
                      void* sf, qg_stream_t stream) {
  if (!x || !q || !sf) return QG_ERR_ARG;
  if (x_dtype != QG_DTYPE_F32 && x_dtype != QG_DTYPE_BF16) return QG_ERR_DTYPE;
  if (layout < QG_LAYOUT_REF_LINEAR || layout > QG_LAYOUT_MMA_KMAJOR) return QG_ERR_LAYOUT;
  if (rows < 1 || k < 32 || (k % 32) != 0) return QG_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(q)) return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (layout != QG_LAYOUT_REF_LINEAR && ((rows % 128) != 0 || ((k / 32) % 4) != 0)) {
    if (cudaMemsetAsync(sf, 0, static_cast<size_t>(qg_scale_bytes(rows, k, 32)), s) != cudaSuccess)
      return QG_ERR_CUDA;
  }
  return launch_quantize_mxfp4(x, x_dtype == QG_DTYPE_BF16, rows, k, layout,
                               static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf),
                               s) == cudaSuccess
             ? QG_OK
             : QG_ERR_CUDA;
}

int qg_gemm_mxfp8(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf, void* c,
                  int c_dtype, int64_t m, int64_t n, int64_t k, int64_t ldc, int sf_layout,
                  uint32_t* status, qg_stream_t stream) {
  return gemm_common(0, a_q, a_sf, nullptr, b_q, b_sf, nullptr, c, c_dtype, m, n, k, ldc,
                     sf_layout, status, reinterpret_cast<cudaStream_t>(stream));
}

// Decode GEMM on CTA pairs for m in (32, 128] at the decode shapes (a build
// with -DQG_SKINNY_PAIR=0 keeps the single-CTA wide tiles, for A/B
// measurement).
#ifndef QG_SKINNY_PAIR
#define QG_SKINNY_PAIR 1
#endif
#ifndef QG_SKINNY_PAIR_QUANT_WIDE
#define QG_SKINNY_PAIR_QUANT_WIDE 1
#endif

// Workspace of qg_gemm_nvfp4_skinny, each part 256-byte aligned: the
// per-CTA partial tiles [max_ctas][2][m][128] fp32, the tile counters
// [tiles][4] (zeroed by the quantiser kernel of every call), the quantised
// activations (values, scales), the tensor scale and the quantiser's per-CTA
// amax slots.
static int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }
struct SkinnyWs {
  int64_t part, cnt, xq, xsf, xts, amax, total;
};
static SkinnyWs skinny_ws_layout(int64_t m, int64_t n, int64_t k) {
  SkinnyWs w;
  const int64_t slices = 2 * skinny_shape(m).halves;
  w.part = 0;
  w.cnt = w.part + align256(static_cast<int64_t>(skinny_max_ctas()) * slices * m * 128 * 4);
  w.xq = w.cnt + align256((n + 255) / 256 * 2 * 4 * 4);  // 4 counters per 128 rows
  w.xsf = w.xq + align256(m * k / 2);
  w.xts = w.xsf + align256(qg_scale_bytes(m, k, 16));
  w.amax = w.xts + 256;
  w.total = w.amax + align256(skinny_max_ctas() * 4);
  return w;
}
size_t qg_gemm_nvfp4_skinny_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m < 1 || n < 1 || k < 1) return 0;
  return static_cast<size_t>(skinny_ws_layout(m, n, k).total);
}

int qg_gemm_nvfp4_skinny(const void* x, int x_dtype, int64_t m, const void* w_q, const void* w_sf,
                         const float* w_ts, void* c, int c_dtype, int64_t n, int64_t k,
                         int64_t ldc, int sf_layout, void* workspace, size_t workspace_bytes,
                         uint32_t* status, qg_stream_t stream) {
  if (!x || !w_q || !w_sf || !c || !workspace) return QG_ERR_ARG;
  if (x_dtype != QG_DTYPE_F32 && x_dtype != QG_DTYPE_BF16) return QG_ERR_DTYPE;
  if (c_dtype != QG_DTYPE_F32 && c_dtype != QG_DTYPE_BF16) return QG_ERR_DTYPE;
  if (sf_layout != QG_LAYOUT_MMA && sf_layout != QG_LAYOUT_MMA_KMAJOR) return QG_ERR_LAYOUT;
  if (m < 1 || m > 128 || n < 1 || k < 32 || (k % 32) != 0 || ldc < n) return QG_ERR_SHAPE;
  if (n > (1ll << 31) - 1 || k > (1ll << 31) - 1) return QG_ERR_SHAPE;
  if (workspace_bytes < qg_gemm_nvfp4_skinny_workspace_bytes(m, n, k)) return QG_ERR_ARG;
  if (!aligned16(x) || !aligned16(w_q) || !aligned16(w_sf) || !aligned16(workspace))
    return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  if (!encode_fn()) return QG_ERR_CUDA;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  const SkinnyWs wl = skinny_ws_layout(m, n, k);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(base + wl.cnt);
  uint8_t* xq = base + wl.xq;
  uint8_t* xsf = base + wl.xsf;
  float* xts = reinterpret_cast<float*>(base + wl.xts);
  const int mma_n = skinny_mma_n(m);
  const SkinnyShape sh = skinny_shape(m);
  // CTA pairs (one whole 512-row weight tile each, half of the activation
  // rows loaded per CTA) when the tiles nearly fill the SMs, as at the
  // decode shapes (n = 28672: 56 pairs on 148 SMs); stream-K otherwise.
  const int64_t pair_tiles = (n + skinny_pair_tile_rows() - 1) / skinny_pair_tile_rows();
  const bool use_pair = QG_SKINNY_PAIR && mma_n >= 64 && 2 * pair_tiles <= num_sms() &&
                        8 * pair_tiles >= 3 * num_sms();
  SkinnyParams p;
  std::memset(&p, 0, sizeof(p));
  const int64_t row_bytes = k / 2;
  if (!make_operand_map(&p.tm_w, w_q, n, row_bytes, 128)) return QG_ERR_CUDA;
  if (!make_operand_map(&p.tm_x, xq, m, row_bytes, use_pair ? mma_n / 2 : mma_n))
    return QG_ERR_CUDA;
  if (!make_scale_map(&p.tm_sfw, w_sf, n, k, 16, sf_layout, 1, sh.sf_chunks)) return QG_ERR_CUDA;
  if (!make_scale_map(&p.tm_sfx, xsf, m, k, 16, QG_LAYOUT_MMA, 1, sh.sf_chunks))
    return QG_ERR_CUDA;
  p.part = reinterpret_cast<float*>(base + wl.part);
  p.cnt = cnt;
  p.c = c;
  p.ldc = ldc;
  p.x = x;
  p.x_bf16 = x_dtype == QG_DTYPE_BF16 ? 1 : 0;
  p.xq = xq;
  p.xsf = xsf;
  p.x_ts = xts;
  p.amax_part = reinterpret_cast<float*>(base + wl.amax);
  p.w_ts = w_ts;
  p.out_bf16 = c_dtype == QG_DTYPE_BF16 ? 1 : 0;
  p.vec_ok = (reinterpret_cast<uintptr_t>(c) % 16 == 0) &&
             ((ldc * (c_dtype == QG_DTYPE_BF16 ? 2 : 4)) % 16 == 0);
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.num_tiles = static_cast<int>((n + sh.tile_rows - 1) / sh.tile_rows);
  p.num_k_blocks = static_cast<int>((row_bytes + sh.stage_k_bytes - 1) / sh.stage_k_bytes);
  p.slices = 2 * sh.halves;
  p.num_counters = p.num_tiles * sh.halves * 4;
  p.status = status;
  p.timeout_ns = default_timeout_ns();
  // Activation quantiser (two small kernels), then the GEMM, which starts
  // streaming weights while they run (programmatic dependent launch).
  const int64_t xblocks = m * (k / 16);
  const int64_t units = static_cast<int64_t>(p.num_tiles) * p.num_k_blocks;
  int64_t grid = units < num_sms() ? units : num_sms();
  // 256-row tiles that nearly fill the SMs (n = 28672: 112 tiles on 148):
  // one whole tile per CTA.  Stream-K over all SMs would leave every tile
  // split and every CTA's last segment a sum of partials after the weight
  // stream (measured 2.5 TB/s against 4.1 at m = 128).
  if (sh.halves == 2 && p.num_tiles <= num_sms() && 4 * p.num_tiles >= 3 * num_sms())
    grid = p.num_tiles;
  if (grid > skinny_max_ctas()) grid = skinny_max_ctas();
  if (use_pair) {
    p.num_tiles = static_cast<int>(pair_tiles);
    p.num_counters = 0;  // no split tiles
    grid = 2 * pair_tiles;
  }
  // Quantiser CTAs (128 threads, <= 56 registers) beside the GEMM's: two fit
  // next to a pair-kernel CTA (<= 112 registers per thread), so for m > 64
  // the quantiser may use up to skinny_max_ctas() CTAs there (at m = 128 two
  // 16-element blocks per thread instead of ~3.5: one load round instead of
  // two).  A/B on one box, GB/s: m = 128 4347 / 4373 / 4357 -> 4517 / 4535 /
  // 4572; m = 64 (one block per thread either way) 4717 / 4737 / 4712 ->
  // 4690 / 4725 / 4705, so m <= 64 keeps one CTA per SM.
  const int quant_ctas =
      use_pair && mma_n == 128 && QG_SKINNY_PAIR_QUANT_WIDE ? skinny_max_ctas() : num_sms();
  if (launch_skinny_quant(p, skinny_quant_grid(xblocks, quant_ctas), s) != cudaSuccess)
    return QG_ERR_CUDA;
  const cudaError_t le = use_pair ? launch_gemm_skinny_pair(p, static_cast<int>(grid), s)
                                  : launch_gemm_skinny(p, static_cast<int>(grid), s);
  if (le != cudaSuccess) return QG_ERR_CUDA;
  return QG_OK;
}

int qg_gemm_nvfp4_gather(const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                         const void* b_sf, const float* b_ts, void* const* c_ranks, int nranks,
                         int64_t col0, int64_t m, int64_t n_local, int64_t k, int64_t ldc,
                         int sf_layout, uint32_t* status, qg_stream_t stream) {
  if (!c_ranks || nranks < 1 || nranks > QG_MAX_RANKS) return QG_ERR_ARG;
  if (col0 < 0 || col0 + n_local > ldc) return QG_ERR_SHAPE;
  Gather g;
  g.c_ranks = c_ranks;
  g.nranks = nranks;
  g.col0 = col0;
  return gemm_common(1, a_q, a_sf, a_ts, b_q, b_sf, b_ts, c_ranks[0], QG_DTYPE_BF16, m,
                     n_local, k, ldc, sf_layout, status, reinterpret_cast<cudaStream_t>(stream), g);
}

// CUDA IPC of device buffers (the fused gather's peer outputs).  The handle
// carries the cudaIpcMemHandle_t of the allocation that holds dptr and
// dptr's offset in it, so buffers from a caching allocator work too.
namespace {
std::mutex g_ipc_mu;
std::map<void*, void*> g_ipc_base;  // imported pointer -> mapped allocation base
}  // namespace

static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(uint64_t) == QG_IPC_HANDLE_BYTES, "IPC handle");

int qg_ipc_export(const void* dptr, void* handle_out) {
  if (!dptr || !handle_out) return QG_ERR_ARG;
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range = [] {
    void* fp = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fp, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<RangeFn>(nullptr);
    return reinterpret_cast<RangeFn>(fp);
  }();
  if (!range) return QG_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dptr)) != CUDA_SUCCESS) return QG_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return QG_ERR_CUDA;
  const uint64_t off = reinterpret_cast<uint64_t>(dptr) - static_cast<uint64_t>(base);
  std::memcpy(handle_out, &h, sizeof(h));
  std::memcpy(static_cast<uint8_t*>(handle_out) + sizeof(h), &off, sizeof(off));
  return QG_OK;
}

int qg_ipc_import(const void* handle, void** dptr_out) {
  if (!handle || !dptr_out) return QG_ERR_ARG;
  cudaIpcMemHandle_t h;
  uint64_t off = 0;
  std::memcpy(&h, handle, sizeof(h));
  std::memcpy(&off, static_cast<const uint8_t*>(handle) + sizeof(h), sizeof(off));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return QG_ERR_CUDA;
  void* p = static_cast<uint8_t*>(base) + off;
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  g_ipc_base[p] = base;
  *dptr_out = p;
  return QG_OK;
}

int qg_ipc_close(void* dptr) {
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    auto it = g_ipc_base.find(dptr);
    if (it == g_ipc_base.end()) return QG_ERR_ARG;
    base = it->second;
    g_ipc_base.erase(it);
  }
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? QG_OK : QG_ERR_CUDA;
}

int qg_read_status(uint32_t* status, uint32_t* device_code, qg_stream_t stream) {
  if (!status) return QG_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, status, sizeof(v), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return QG_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return QG_ERR_CUDA;
  if (cudaMemsetAsync(status, 0, sizeof(uint32_t), s) != cudaSuccess) return QG_ERR_CUDA;
  if (device_code) *device_code = v;
  return v == 0 ? QG_OK : QG_ERR_TIMEOUT;
}

int qg_selftest_e2m1_cvt(unsigned long long* out, qg_stream_t stream) {
  if (!out) return QG_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return QG_ERR_ALIGN;
  if (int d = check_device()) return d;
  return launch_e2m1_cvt_selftest(out, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
             ? QG_OK
             : QG_ERR_CUDA;
}

int qg_selftest_wait_timeout(uint64_t timeout_ns, uint32_t* status, qg_stream_t stream) {
  if (!status) return QG_ERR_ARG;
  if (timeout_ns > 1000000000ull) return QG_ERR_ARG;  // keep the self test short
  if (int d = check_device()) return d;
  return launch_wait_timeout_selftest(timeout_ns, status, reinterpret_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? QG_OK
             : QG_ERR_CUDA;
}

}  // extern "C"
