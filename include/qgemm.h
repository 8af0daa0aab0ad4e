/* qgemm.h -- C ABI of the B200 (sm_100a) block-scaled quantized GEMM library.
 *
 * This is the drop-in boundary for the reference's quant-GEMM path
 * (hibouwu/CUDA_optimazation).  The reference has no in-process API: its
 * operator surface is the NVFP4 host quantizer
 * (GEMMsm110/include/requant/nvfp4_reference.cuh:76-112), the device requant
 * primitives (GEMMsm110/include/requant/sm110_tcgen05_epilogue.cuh:75-160),
 * the tc6 runner (GEMMsm110/include/backends/tc6_nvfp4.cuh:561-619) and the
 * CUTLASS 72b NVFP4 backend the harness shells out to
 * (GEMMquant_sm110/build_and_run.sh:38-75).  Each entry point below names the
 * reference interface it replaces.
 *
 * Conventions
 *  - Every pointer is caller-owned DEVICE memory unless stated otherwise.
 *    No entry point allocates device memory.
 *  - Calls are stream-ordered and asynchronous: a QG_OK return means the
 *    work was enqueued on `stream`.  Device-side failures (a bounded wait that
 *    timed out) are reported through `status` words read by qg_read_status().
 *  - Nothing here calls exit() or abort().
 *  - Operands are K-major: A is M x K row-major, B is N x K row-major
 *    ("B^T" layout), C = A * B^T is M x N row-major with leading dimension ldc.
 */
#ifndef QGEMM_B200_H
#define QGEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qg_stream_t; /* == cudaStream_t; NULL = legacy stream */

typedef enum {
  QG_OK = 0,
  QG_ERR_SHAPE = 1,       /* M, N or K out of the supported range          */
  QG_ERR_ALIGN = 2,       /* pointer / leading dimension not 16-B aligned   */
  QG_ERR_LAYOUT = 3,      /* layout not accepted by this entry point        */
  QG_ERR_DTYPE = 4,       /* unknown dtype code                             */
  QG_ERR_CUDA = 5,        /* a CUDA runtime / driver call failed            */
  QG_ERR_TIMEOUT = 6,     /* a device wait exceeded its bound (status word) */
  QG_ERR_ARG = 7,         /* null pointer or bad argument                   */
  QG_ERR_UNSUPPORTED = 8  /* device is not sm_100                           */
} qg_status;

typedef enum { QG_DTYPE_F32 = 0, QG_DTYPE_BF16 = 1 } qg_dtype;

/* Operand layouts.
 *  QG_LAYOUT_REF_LINEAR : the reference quantizer's byte order
 *      (nvfp4_reference.cuh:76-112): the tensor is flattened row-major, value
 *      2i goes to the HIGH nibble of byte i (pack_fp4.cuh:11-15), and one
 *      scale byte per 16 flattened elements in linear order.
 *  QG_LAYOUT_MMA : the tensor-core operand order: row-major, value 2i in
 *      the LOW nibble, scales in 512-byte chunks of 128 rows x 4 scale columns
 *      at cutlass-gemm-cpp-guide/include/guide/scale_layout.hpp:11-26
 *      (chunk index = scale_block * row_blocks + row_block).
 *  QG_LAYOUT_MMA_KMAJOR : as QG_LAYOUT_MMA, but chunks of one 128-row block
 *      are contiguous along K (chunk index = row_block * scale_blocks +
 *      scale_block), the order CUTLASS's Sm1xxBlockScaledConfig
 *      tile_to_shape(..., Step<_2,_1>) produces.  The two MMA orders coincide
 *      when either block count is 1.
 */
typedef enum {
  QG_LAYOUT_REF_LINEAR = 0,
  QG_LAYOUT_MMA = 1,
  QG_LAYOUT_MMA_KMAJOR = 2
} qg_layout;

/* Human-readable name of a qg_status code. */
const char* qg_status_string(int status);

/* Library version string. */
const char* qg_version(void);

/* Bytes of the scale-factor buffer for an MN x K operand with one scale per
 * `sv` K elements (16 for NVFP4, 32 for MXFP8) in an MMA layout:
 * ceil(MN/128) * ceil(ceil(K/sv)/4) * 512.
 * Replaces guide::sm1xx_scale_storage_size (scale_layout.hpp:28-34). */
int64_t qg_scale_bytes(int64_t mn, int64_t k, int sv);

/* Workspace bytes qg_quantize_nvfp4 needs (one amax word, padded). */
size_t qg_quantize_workspace_bytes(void);

/* NVFP4 quantizer: x (rows x k, fp32 or bf16, row-major) -> e2m1 values `q`
 * (rows*k/2 bytes), e4m3 block scales `sf` (one per 16 K elements; in
 * QG_LAYOUT_REF_LINEAR rows*k/16 bytes, else qg_scale_bytes(rows, k, 16)
 * bytes) and the fp32 tensor scale *ts = amax / (448 * 6) (1 if amax == 0).
 * Bit-exact to make_nvfp4_reference (nvfp4_reference.cuh:76-112), which this
 * replaces together with the device twins sm110_make_nvfp4_block_scale /
 * sm110_requant_nvfp4_e2m1x2 (sm110_tcgen05_epilogue.cuh:75-160).
 * REF_LINEAR accepts any rows*k; the MMA layouts need k % 16 == 0.
 * `workspace` (device, qg_quantize_workspace_bytes()) holds the amax scratch
 * word and is cleared on `stream` by the call. */
int qg_quantize_nvfp4(const void* x, int x_dtype, int64_t rows, int64_t k, int layout, void* q,
                      void* sf, float* ts, void* workspace, qg_stream_t stream);

/* qg_quantize_nvfp4 without the workspace argument, for callers that cannot
 * allocate device memory: plugins hosted by a framework that owns every
 * device allocation and hands over only the call's tensors, allocator-free
 * embedded runtimes, code called back from inside a memory allocator, and
 * latency-critical loops that cannot afford cudaMalloc's implicit device
 * synchronisation.  No counterpart in the reference.  Same outputs as
 * qg_quantize_nvfp4, bit for bit.  Its scratch is a fixed 64.25 KiB array in
 * the library's device memory (held by every GPU that loads the library until
 * exit), which bounds the input to qg_quantize_nvfp4_noalloc_max_elements()
 * = 2^28 elements; larger inputs return QG_ERR_SHAPE.  The array's device
 * address is looked up on the first call on each device, so make that first
 * call before any stream capture.  A device reset (cudaDeviceReset) moves
 * the array: the first call after it fails with QG_ERR_CUDA and forgets the
 * cached address, and the next call looks it up again.  An error already
 * pending in the CUDA runtime before the call is reported as QG_ERR_CUDA
 * without launching and is left pending.  All calls share the array: calls
 * that may overlap on the GPU race and must be ordered by the caller.
 * Allocates nothing (no cudaMalloc / cudaFree, no allocating library
 * routine). */
int qg_quantize_nvfp4_noalloc(const void* x, int x_dtype, int64_t rows, int64_t k, int layout,
                              void* q, void* sf, float* ts, qg_stream_t stream);

/* Largest rows * k qg_quantize_nvfp4_noalloc accepts. */
int64_t qg_quantize_nvfp4_noalloc_max_elements(void);

/* MXFP8 quantizer (OCP MX v1.0; the reference has none): x (rows x k) ->
 * e4m3 values `q` (rows*k bytes) and ue8m0 scales per 32 K elements, scale
 * exponent floor(log2(block amax)) - 8 clamped to [-127, 127] (all-zero
 * blocks get code 0).  k % 32 == 0.  Layout REF_LINEAR writes the scales as
 * [rows][k/32]; the MMA layouts as qg_scale_bytes(rows, k, 32) bytes. */
int qg_quantize_mxfp8(const void* x, int x_dtype, int64_t rows, int64_t k, int layout, void* q,
                      void* sf, qg_stream_t stream);

/* MXFP4 quantizer (OCP MX v1.0 with E2M1 elements; the reference has no
 * MXFP4 quantizer, its MXFP4 rows run CUTLASS example 72a with
 * mx_float4_t, GEMMquant_sm110/build_and_run.sh:77-115): x (rows x k) ->
 * e2m1 values `q` (rows*k/2 bytes) and ue8m0 scales per 32 K elements,
 * scale exponent floor(log2(block amax)) - 2 clamped to [-127, 127]
 * (all-zero blocks get code 0), elements e2m1 round-to-nearest-even of
 * x * 2^-e, saturating at 6, NaN -> +0.  k % 32 == 0.  Layout REF_LINEAR
 * packs the first element of each pair in the HIGH nibble and writes the
 * scales as [rows][k/32]; the MMA layouts pack low nibble first with
 * qg_scale_bytes(rows, k, 32) scale bytes. */
int qg_quantize_mxfp4(const void* x, int x_dtype, int64_t rows, int64_t k, int layout, void* q,
                      void* sf, qg_stream_t stream);

/* Re-lay an NVFP4 operand between layouts (rows x k, k % 16 == 0).  Source
 * and destination must not alias. */
int qg_repack_nvfp4(const void* src_q, const void* src_sf, int src_layout, void* dst_q,
                    void* dst_sf, int dst_layout, int64_t rows, int64_t k, qg_stream_t stream);

/* Re-lay an MX operand (one ue8m0 scale per 32 K elements) between layouts:
 * elem_bits 4 (MXFP4: nibble order flipped between REF_LINEAR and the MMA
 * layouts) or 8 (MXFP8: value bytes unchanged).  rows x k, k % 32 == 0,
 * value buffers 16-byte aligned; source and destination must not alias.
 * Used by the quantised-weight file tool (cuda_optimazation_b200/weights.py)
 * so stored weights load in either layout without re-quantising.  No
 * reference counterpart (the reference stores no quantised weights;
 * Nvfp4ReferenceResult, nvfp4_reference.cuh:18-22, is its in-memory form). */
int qg_repack_mx(int elem_bits, const void* src_q, const void* src_sf, int src_layout,
                 void* dst_q, void* dst_sf, int dst_layout, int64_t rows, int64_t k,
                 qg_stream_t stream);

/* NVFP4 x NVFP4 block-scaled GEMM on tcgen05 (kind::mxf4nvf4, block16):
 *   C[m, n] = (a_ts * b_ts) * sum_k a(m,k) sfa(m,k/16) b(n,k) sfb(n,k/16)
 * a_q / b_q in the MMA nibble order (M*K/2 and N*K/2 bytes), scales in
 * `sf_layout` (QG_LAYOUT_MMA or QG_LAYOUT_MMA_KMAJOR); a_ts / b_ts point at
 * one device float each (NULL = 1.0).  c_dtype fp32 or bf16, ldc >= n
 * (elements).  K % 32 == 0; M, N >= 1.  `status` (device uint32, may be
 * NULL) receives a nonzero QG device code if a bounded wait expired.
 * Replaces the CUTLASS 72b NVFP4 GEMM backend (build_and_run.sh:38-75) and
 * the planned nvfp4_q1_native_fp4_mainloop slot
 * (GEMMquant_sm110/scripts/run_quant_gemm_1024.py:37-43). */
int qg_gemm_nvfp4(const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                  const void* b_sf, const float* b_ts, void* c, int c_dtype, int64_t m, int64_t n,
                  int64_t k, int64_t ldc, int sf_layout, uint32_t* status, qg_stream_t stream);

/* NVFP4 GEMM whose output is NVFP4: the epilogue requantises each
 * 16-column block of every output row to e2m1 values plus one e4m3 scale,
 * instead of storing bf16 / fp32.  The element values are the fp32 numbers
 * qg_gemm_nvfp4 would store (alpha = a_ts * b_ts applied), quantised with
 * the steps of make_nvfp4_reference (nvfp4_reference.cuh:76-112) under the
 * caller's tensor scale *out_ts (device float; NULL = 1.0): for every block,
 * s = e4m3_round_up(max|v / ts| / 6), q = e2m1(v * ((1/ts) / s)).  The
 * result is therefore bit-identical to qg_quantize_nvfp4's block step
 * applied to qg_gemm_nvfp4's fp32 output with the same tensor scale.
 * out_q receives m*n/2 bytes, out_sf the scales in out_layout
 * (QG_LAYOUT_REF_LINEAR: m*n/16 bytes in flat order, high nibble first, the
 * reference's layout; an MMA layout: qg_scale_bytes(m, n, 16) bytes, low
 * nibble first, so the output feeds the next GEMM as its A operand with
 * K = n).  out_amax (device uint32, may be NULL) is max-reduced with the
 * bit pattern of max|v| over the outputs (a float; the caller zeroes it), so
 * the next call's tensor scale can be amax / 2688.  n % 16 == 0, out_q 16-B
 * and out_sf 4-B aligned; other rules as qg_gemm_nvfp4.
 * Replaces the tc6 fused NVFP4 epilogue (Tc6Runner and store_tile,
 * GEMMsm110/include/backends/tc6_nvfp4.cuh:460-503, :561-619), which takes
 * the inverse tensor scale as an argument in the same way. */
int qg_gemm_nvfp4_requant(const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                          const void* b_sf, const float* b_ts, const float* out_ts, void* out_q,
                          void* out_sf, int out_layout, uint32_t* out_amax, int64_t m, int64_t n,
                          int64_t k, int sf_layout, uint32_t* status, qg_stream_t stream);

/* MXFP8 x MXFP8 block-scaled GEMM on tcgen05 (kind::mxf8f6f4, ue8m0 per 32
 * K): C = sum_k a*sfa*b*sfb.  a_q / b_q are e4m3 bytes (M*K, N*K), K % 32
 * == 0.  Replaces the unscaled FP8 stages fp8_q0..q8
 * (GEMMquant_sm110/src/quant_gemm_bench.cu:285-662, :1314-1373) with the
 * scaled format of cutlass-gemm-cpp-guide/cases/bs_mxfp8_1sm_p128. */
int qg_gemm_mxfp8(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf, void* c,
                  int c_dtype, int64_t m, int64_t n, int64_t k, int64_t ldc, int sf_layout,
                  uint32_t* status, qg_stream_t stream);

/* MXFP4 x MXFP4 block-scaled GEMM on tcgen05 (kind::mxf4nvf4.block32,
 * ue8m0 scale per 32 K): C = sum_k a*sfa*b*sfb.  a_q / b_q are e2m1 codes
 * in the MMA nibble order (M*K/2, N*K/2 bytes), scales in sf_layout (an MMA
 * layout, qg_scale_bytes(rows, K, 32) bytes).  K % 32 == 0; rules otherwise
 * as qg_gemm_nvfp4.  Replaces the CUTLASS 72a MXFP4 backend rows
 * mxfp4_q0_cutlass_72a_mxfp4_bf16 / mxfp4_q1_cutlass_72a_swizzle1
 * (GEMMquant_sm110/scripts/run_quant_gemm_1024.py:54-73). */
int qg_gemm_mxfp4(const void* a_q, const void* a_sf, const void* b_q, const void* b_sf, void* c,
                  int c_dtype, int64_t m, int64_t n, int64_t k, int64_t ldc, int sf_layout,
                  uint32_t* status, qg_stream_t stream);

/* ---- Plans: the host work of a GEMM call done once --------------------
 * A plan binds one GEMM call -- operands, output, shapes, layout -- and
 * does its host work once: argument checks, TMA tensor-map encodes, kernel
 * and grid choice.  qg_plan_run() then only enqueues the kernel, for loops
 * that repeat the same call (a decode step, a layer) on buffers whose
 * contents change between runs.  A plan lives in host memory (no device
 * allocation), belongs to the device current at creation (run it with that
 * device current) and reads the operands at run time, not at creation.
 * format: QG_FORMAT_NVFP4 (a_ts / b_ts as qg_gemm_nvfp4), QG_FORMAT_MXFP8,
 * QG_FORMAT_MXFP4 (tensor scales ignored); other arguments and rules as
 * the matching qg_gemm_* entry point.  No reference counterpart (the
 * reference's runners re-create their state per launch). */
typedef struct qg_plan_st* qg_plan;
typedef enum { QG_FORMAT_MXFP8 = 0, QG_FORMAT_NVFP4 = 1, QG_FORMAT_MXFP4 = 2 } qg_format;
int qg_plan_create_gemm(qg_plan* plan, int format, const void* a_q, const void* a_sf,
                        const float* a_ts, const void* b_q, const void* b_sf, const float* b_ts,
                        void* c, int c_dtype, int64_t m, int64_t n, int64_t k, int64_t ldc,
                        int sf_layout, uint32_t* status);
int qg_plan_run(qg_plan plan, qg_stream_t stream);
int qg_plan_destroy(qg_plan plan);

/* Decode-shaped NVFP4 GEMM with the activation quantisation fused into the
 * call: x (m x k, bf16 or fp32, m <= 128) is quantised to NVFP4 exactly as
 * qg_quantize_nvfp4 would, then C[m, n] = (ts_x * w_ts) * x_q . w_q^T with the
 * pre-quantised weights w_q (n x k, MMA layout, scales in sf_layout).  The
 * weights are streamed once from HBM: stream-K over 128-row weight tiles
 * (256-row tiles of two halves for m > 32) on every SM, or, for m in
 * (32, 128] when n's 512-row tiles nearly fill the SMs (decode shapes such
 * as n = 28672), one whole tile per CTA pair (a thread-block cluster of two)
 * with each CTA loading half of the activation rows.  Three launches on
 * `stream`: an amax pass over x, the
 * quantiser, and the GEMM, the last two with programmatic dependent launch so
 * the GEMM streams weights while x is quantised.  `workspace` (device,
 * qg_gemm_nvfp4_skinny_workspace_bytes) holds the partial tiles, the
 * quantised activations and the tile counters; it needs no initialisation
 * (every call rewrites what it reads, counters and scale padding included,
 * also after a call that returned a device timeout).  One workspace serves
 * one stream at a time.  K % 32 == 0.  The result is
 * deterministic (split tiles are summed in a fixed order; pair tiles are
 * never split).
 * No reference counterpart kernel: the reference harness runs square
 * problems only (GEMMquant_sm110/src/quant_gemm_bench.cu:3038-3079); this is
 * the decode configuration of its quant-GEMM path. */
int qg_gemm_nvfp4_skinny(const void* x, int x_dtype, int64_t m, const void* w_q, const void* w_sf,
                         const float* w_ts, void* c, int c_dtype, int64_t n, int64_t k,
                         int64_t ldc, int sf_layout, void* workspace, size_t workspace_bytes,
                         uint32_t* status, qg_stream_t stream);

/* Workspace bytes qg_gemm_nvfp4_skinny needs. */
size_t qg_gemm_nvfp4_skinny_workspace_bytes(int64_t m, int64_t n, int64_t k);

/* ---- Column-parallel GEMM with the output all-gather fused in ----------
 * BASELINE config 5 shards B along N over the GPUs of one box
 * (GEMMquant_sm110 itself is single-GPU; the north star asks for the N-sharded
 * split with an optional output all-gather).  Instead of a GEMM followed by
 * a collective, the CTA-pair GEMM's epilogue TMA-stores every output box
 * into the C buffer of EVERY rank, so the NVLink transfer overlaps the math
 * tile by tile.
 *
 * c_ranks[r] (r < nranks <= QG_MAX_RANKS) is rank r's full bf16 C (m rows,
 * row stride ldc elements), this process's own buffer included; peers'
 * buffers are mapped with qg_ipc_import.  This call computes
 * C[:, col0 : col0 + n_local] = (a_ts*b_ts) * A . B_local^T (B_local: the
 * n_local rows of B this rank owns, NVFP4, MMA layout) and writes those
 * columns into every c_ranks[r].  col0 % 8 == 0, ldc % 8 == 0, buffers
 * 16-byte aligned.  Stream-ordered on this GPU only, and every rank's call
 * writes into every rank's C, so the caller orders the ranks on both sides:
 * after the calls (synchronise + a host barrier) before reading the
 * gathered C, and before the next calls (every rank done reading its C,
 * on any stream: synchronise + a host barrier), or a fast peer overwrites a
 * result still being read.  colpar.colpar_gemm_fused does both. */
#define QG_MAX_RANKS 8
int qg_gemm_nvfp4_gather(const void* a_q, const void* a_sf, const float* a_ts, const void* b_q,
                         const void* b_sf, const float* b_ts, void* const* c_ranks, int nranks,
                         int64_t col0, int64_t m, int64_t n_local, int64_t k, int64_t ldc,
                         int sf_layout, uint32_t* status, qg_stream_t stream);

/* CUDA IPC for the gather's peer buffers.  A handle is QG_IPC_HANDLE_BYTES:
 * the cudaIpcMemHandle_t of the allocation holding dptr plus dptr's offset
 * in it (so pointers inside a caching allocator's block work).  Import maps
 * a peer's buffer into this process (peer access enabled lazily); close
 * unmaps it.  No reference counterpart. */
#define QG_IPC_HANDLE_BYTES 72
int qg_ipc_export(const void* dptr, void* handle_out);
int qg_ipc_import(const void* handle, void** dptr_out);
int qg_ipc_close(void* dptr);

/* Read and clear a device status word (synchronises `stream`).  Returns
 * QG_OK, QG_ERR_TIMEOUT or QG_ERR_CUDA; *device_code (may be NULL) gets the
 * raw device code. */
int qg_read_status(uint32_t* status, uint32_t* device_code, qg_stream_t stream);

/* Exhaustive self test of the hardware e2m1 conversion that the
 * requantising GEMM epilogue uses (cvt.rn.satfinite.e2m1x2.f32) against the
 * library's restatement of the reference encoder encode_e2m1_rn
 * (GEMMsm110/include/requant/e2m1_encode.cuh:18-44), over all 2^32 fp32 bit
 * patterns.  out (device, 3 x uint64, written on `stream`): [0] mismatches on
 * non-NaN inputs (must be 0), [1] mismatches on NaN inputs (the epilogue maps
 * NaN to +0 itself), [2] largest mismatching non-NaN pattern + 1. */
int qg_selftest_e2m1_cvt(unsigned long long* out, qg_stream_t stream);

/* Failure-path self test: launches one CTA that waits on an mbarrier no one
 * arrives on, bounded by `timeout_ns`, and records the timeout in *status.
 * Exists so tests can prove the bounded-wait path returns QG_ERR_TIMEOUT
 * without hanging the GPU.  No reference counterpart (its waits are
 * unbounded, GEMMsm110/include/sm110_ptx_helpers.cuh:77-91). */
int qg_selftest_wait_timeout(uint64_t timeout_ns, uint32_t* status, qg_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* QGEMM_B200_H */
