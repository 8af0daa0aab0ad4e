// qg_gemm.h -- internal launch interface between the C-ABI host code and
// the kernels.  Not part of the public ABI (include/qgemm.h is).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace qg {

// Devices a process may drive (per-device launch state is kept in arrays).
constexpr int kMaxDevices = 64;

// Diagnostic switches, fixed when the library is compiled (-DQG_DIAG_FLAGS=...
// through QG_EXTRA_NVCC); shipped builds have none and the branches vanish.
// Results are wrong by design when any of bits 0-3, 7, 8, 11 is set:
// bit 0 skips the scale staging, bit 1 the MMAs, bit 2 the TMA loads (pair /
// solo kernels), bit 3 the epilogue stores, bit 7 the pair kernel's B loads,
// bit 8 its SFB loads, bit 11 all its scale loads and their shared memory.
// Bit 6 makes the decode GEMM's CTA (kDiag >> 16) and its quantiser kernels
// write %globaltimer stamps of their roles, and every decode GEMM CTA its
// start, end and epilogue milestones (into an unused partial slice); bit 9
// makes the pair kernel's first pair stamp its roles into C.  Used to
// attribute kernel time to its parts.
#ifndef QG_DIAG_FLAGS
#define QG_DIAG_FLAGS 0u
#endif
constexpr uint32_t kDiag = QG_DIAG_FLAGS;

struct GemmParams {
  CUtensorMap tm_a;    // uint8 [rows][K bytes], box 128 B x kBM, SWIZZLE_128B
  CUtensorMap tm_b;    // uint8 [rows][K bytes], box 128 B x kBN, SWIZZLE_128B
  CUtensorMap tm_sfa;  // uint32 [scale_blocks][row_blocks][128], box (128, kBM/128, chunks)
  CUtensorMap tm_sfb;
  // bf16 C through TMA stores (pair kernel): box 64 x 32, SWIZZLE_128B.
  // n_out destinations receive the same tile: this GPU's C, or for the
  // fused column-parallel gather every rank's C (peer buffers mapped with
  // CUDA IPC).  n_out == 0: direct stores to c.
  static constexpr int kMaxOut = 8;
  CUtensorMap tm_out[kMaxOut];
  int n_out;
  void* c;
  int64_t ldc;  // elements
  int m, n, k;
  int num_m_tiles, num_n_tiles, num_k_blocks;
  int vec_ok;  // 16-byte vector stores are legal for every full 32-column run
  const float* a_ts;
  const float* b_ts;
  // NVFP4 output (requantising epilogue, pair kernel): values [m][n/2] and
  // one e4m3 scale per 16 columns in layout rq_layout (REF_LINEAR or an MMA
  // order with rq_row_blocks x rq_sf_blocks chunks), decoded with the tensor
  // scale *rq_ts; the output's amax is max-reduced into *rq_amax (optional).
  uint8_t* rq_q;
  uint8_t* rq_sf;
  const float* rq_ts;
  uint32_t* rq_amax;
  int rq_layout;
  int rq_row_blocks, rq_sf_blocks;
  uint32_t* status;
  uint64_t timeout_ns;
};

// Decode-shaped NVFP4 GEMM (gemm_skinny.cu): weights W [n][k] on the MMA's M
// side, activations X [m][k] (m <= 128) on its N side, stream-K over
// (weight tile, K block) units.  The activations are quantised by two small
// kernels launched ahead of it (launch_skinny_quant) with programmatic
// dependent launch, so the GEMM streams weights meanwhile.  A tile split
// between CTAs is summed by the last contributor to finish it (per-tile
// counters), in a fixed order, from per-CTA partial slices; whole tiles are
// written straight to C.
struct SkinnyParams {
  CUtensorMap tm_w;    // uint8 [n][k/2], box 128 B x 128 rows, SWIZZLE_128B
  CUtensorMap tm_x;    // uint8 [m][k/2] (the quantised xq), box 128 B x mma_n rows
  CUtensorMap tm_sfw;  // uint32 chunks, box (128, 1, 4)
  CUtensorMap tm_sfx;
  const void* x;       // activations, fp32 or bf16 [m][k]
  int x_bf16;
  uint8_t* xq;         // quantised activations [m][k/2]
  uint8_t* xsf;        // their scales, MMA layout
  float* x_ts;         // their tensor scale
  float* amax_part;    // [quantiser grid] per-CTA amax
  float* part;         // [grid][2][m][128] fp32 partial tiles
  uint32_t* cnt;       // [num_tiles][4] tile arrival counters, zeroed by the quantiser
  void* c;
  int64_t ldc;
  const float* w_ts;   // weight tensor scale (may be null)
  int out_bf16;
  int vec_ok;          // C rows start 16-byte aligned (16-byte stores legal)
  int m, n, k;
  int num_tiles, num_k_blocks;  // tiles of SkinnyShape::tile_rows, K blocks per stage
  int slices;                    // partial slices per CTA (2 per 128-row half)
  int num_counters;              // words of cnt the quantiser zeroes
  uint32_t* status;
  uint64_t timeout_ns;
};
// Tile geometry of the decode GEMM for m activation rows.
struct SkinnyShape {
  int tile_rows;      // weight rows per tile (128, or 256 as two halves)
  int stage_k_bytes;  // K bytes per stage (256 or 128)
  int sf_chunks;      // 64-K scale chunks per stage
  int halves;         // 128-row halves per tile
};
SkinnyShape skinny_shape(int64_t m);
cudaError_t launch_gemm_skinny(const SkinnyParams& p, int grid, cudaStream_t stream);
// Decode GEMM on CTA pairs (gemm_skinny_pair.cu), MMA N = 64 or 128: one whole
// skinny_pair_tile_rows()-row weight tile per pair (grid = 2 x tiles); tm_x
// has a box of mma_n / 2 rows (each CTA loads half of the activation rows).
cudaError_t launch_gemm_skinny_pair(const SkinnyParams& p, int grid, cudaStream_t stream);
int skinny_pair_tile_rows();
int skinny_quant_grid(int64_t xblocks, int sms);
cudaError_t launch_skinny_quant(const SkinnyParams& p, int grid, cudaStream_t stream);
int skinny_max_ctas();
int skinny_mma_n(int64_t m);

cudaError_t launch_gemm_blockscaled(const GemmParams& p, bool fp4, bool out_bf16, int grid,
                                    cudaStream_t stream);
// fmt: 0 MXFP8, 1 NVFP4, 2 MXFP4.  out_kind: 0 fp32 C, 1 bf16 C, 2 NVFP4
// output (rq_* fields; NVFP4 only), 3 bf16 C through TMA stores (n_out > 0)
// with eight epilogue warps.
cudaError_t launch_gemm_pair(const GemmParams& p, int fmt, int out_kind, int grid,
                             cudaStream_t stream);
int pair_sf_chunks_per_stage(int fmt);
cudaError_t launch_gemm_solo(const GemmParams& p, bool fp4, bool out_bf16, int grid,
                             cudaStream_t stream);
int pair_tile_m();
int pair_tile_n();
int gemm_tile_m();
int gemm_tile_n();
int gemm_stage_k_bytes();
int gemm_sf_chunks_per_stage(bool fp4);

// Quantizer launches (quantize.cu).
cudaError_t launch_amax(const void* x, bool bf16, int64_t n, uint32_t* amax_bits,
                        cudaStream_t stream);
cudaError_t launch_quantize_nvfp4(const void* x, bool bf16, int64_t rows, int64_t k, int layout,
                                  uint8_t* q, uint8_t* sf, float* ts, const uint32_t* amax_bits,
                                  cudaStream_t stream);
cudaError_t launch_quantize_mxfp8(const void* x, bool bf16, int64_t rows, int64_t k, int layout,
                                  uint8_t* q, uint8_t* sf, cudaStream_t stream);
cudaError_t launch_quantize_mxfp4(const void* x, bool bf16, int64_t rows, int64_t k, int layout,
                                  uint8_t* q, uint8_t* sf, cudaStream_t stream);
cudaError_t launch_repack_nvfp4(const uint8_t* sq, const uint8_t* ssf, int src_layout,
                                uint8_t* dq, uint8_t* dsf, int dst_layout, int64_t rows,
                                int64_t k, cudaStream_t stream);
cudaError_t launch_repack_mx(bool fp4, const uint8_t* sq, const uint8_t* ssf, int src_layout,
                             uint8_t* dq, uint8_t* dsf, int dst_layout, int64_t rows, int64_t k,
                             cudaStream_t stream);
cudaError_t launch_e2m1_cvt_selftest(unsigned long long* out, cudaStream_t stream);
cudaError_t launch_wait_timeout_selftest(uint64_t timeout_ns, uint32_t* status,
                                         cudaStream_t stream);

int num_sms();

}  // namespace qg
