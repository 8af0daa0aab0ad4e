// quantize_noalloc.cu -- NVFP4 quantizer entry point that allocates nothing.
//
// Some callers cannot call cudaMalloc at all: plugins hosted by a framework
// that owns every device allocation and hands out only the tensors of a
// call, allocator-free embedded runtimes, code called back from inside a
// memory allocator (re-entering it would deadlock), and latency-critical
// loops that cannot afford cudaMalloc's implicit device synchronisation.
// qg_quantize_nvfp4 needs a caller-provided scratch workspace for its amax
// reduction; such callers may have no way to provide one.  This variant keeps
// that scratch in a fixed array in the library's own device memory instead.
//
// Scratch: a file-scope __device__ array of kNoAllocPartials + 64 words
// (64.25 KiB).  Every GPU that loads this library holds it until the process
// exits.  The amax is reduced in two steps without atomics: each CTA of the
// first kernel writes the maximum of one kChunk-element slice to its own
// slot, a one-CTA kernel folds the slots into the final word, and the
// quantize kernel of qg_quantize_nvfp4 reads that word.  Every slot a call
// reads is written earlier in the same call, so nothing needs clearing.
// Inputs above kNoAllocPartials * kChunk elements do not fit and are rejected.
//
// All calls on a device share the one array and it keeps the last call's
// contents: calls that overlap on the GPU (different streams without
// ordering between them) race on it and must be serialised by the caller.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/qgemm.h"
#include "qg_gemm.h"

namespace qg {

namespace {

constexpr int64_t kChunk = 16384;             // input elements per partial slot
constexpr int64_t kNoAllocPartials = 16384;   // slots -> max 2^28 elements
constexpr int64_t kFinalSlot = kNoAllocPartials;

static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocPartials + 64];

template <bool kBf16>
__global__ void __launch_bounds__(256)
    amax_partial_kernel(const void* x, int64_t n, uint32_t* partials) {
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * kChunk;
  const int64_t end = begin + kChunk < n ? begin + kChunk : n;
  float m = 0.0f;
  if (kBf16) {
    const uint16_t* p = reinterpret_cast<const uint16_t*>(x);
    for (int64_t i = begin + threadIdx.x * 8; i < end; i += 256 * 8) {
      if (i + 8 <= end) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p + i));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          m = fmaxf(m, fabsf(__uint_as_float(w[j] << 16)));
          m = fmaxf(m, fabsf(__uint_as_float(w[j] & 0xffff0000u)));
        }
      } else {
        for (int64_t t = i; t < end; ++t)
          m = fmaxf(m, fabsf(__uint_as_float(static_cast<uint32_t>(p[t]) << 16)));
      }
    }
  } else {
    const float* p = reinterpret_cast<const float*>(x);
    for (int64_t i = begin + threadIdx.x * 4; i < end; i += 256 * 4) {
      if (i + 4 <= end) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p + i));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      } else {
        for (int64_t t = i; t < end; ++t) m = fmaxf(m, fabsf(p[t]));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = red[0];
    for (int i = 1; i < 8; ++i) r = fmaxf(r, red[i]);
    partials[blockIdx.x] = __float_as_uint(r);
  }
}

__global__ void __launch_bounds__(1024) amax_finalize_kernel(uint32_t* scratch, int nparts) {
  uint32_t m = 0u;  // non-negative floats order like their bit patterns
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) m = max(m, scratch[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ uint32_t red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t r = 0u;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) r = max(r, red[i]);
    scratch[kFinalSlot] = r;
  }
}

// Device address of the scratch array, looked up on the first call on each
// device with that device current; in host code the symbol is only a
// stand-in, never a device address.  Because the first call does this
// set-up, make it before any stream capture.  A device reset reloads the
// module and moves the array, so a call whose launches fail forgets the
// cached address and the next call looks it up again.
std::mutex g_scratch_mu;
uint32_t* g_scratch_addr[64] = {nullptr};

void forget_scratch_address() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  g_scratch_addr[dev] = nullptr;
}

uint32_t* scratch_address(int* err) {
  auto& mu = g_scratch_mu;
  auto& addr = g_scratch_addr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = QG_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      *err = QG_ERR_CUDA;
      return nullptr;
    }
    addr[dev] = static_cast<uint32_t*>(p);
  }
  return addr[dev];
}

}  // namespace

}  // namespace qg

using namespace qg;

extern "C" {

int64_t qg_quantize_nvfp4_noalloc_max_elements(void) { return kNoAllocPartials * kChunk; }

int qg_quantize_nvfp4_noalloc(const void* x, int x_dtype, int64_t rows, int64_t k, int layout,
                              void* q, void* sf, float* ts, qg_stream_t stream) {
  if (!x || !q || !sf) return QG_ERR_ARG;
  if (x_dtype != QG_DTYPE_F32 && x_dtype != QG_DTYPE_BF16) return QG_ERR_DTYPE;
  if (layout < QG_LAYOUT_REF_LINEAR || layout > QG_LAYOUT_MMA_KMAJOR) return QG_ERR_LAYOUT;
  if (rows < 1 || k < 1) return QG_ERR_SHAPE;
  if (rows > kNoAllocPartials * kChunk / k) return QG_ERR_SHAPE;  // over the scratch capacity
  if (layout != QG_LAYOUT_REF_LINEAR && (k % 16) != 0) return QG_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(q) & 15u))
    return QG_ERR_ALIGN;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return QG_ERR_CUDA;
  if (major != 10) return QG_ERR_UNSUPPORTED;
  int err = QG_OK;
  uint32_t* scratch = scratch_address(&err);
  if (!scratch) return err;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n = rows * k;
  const bool bf16 = x_dtype == QG_DTYPE_BF16;
  if (layout != QG_LAYOUT_REF_LINEAR && ((rows % 128) != 0 || ((k / 16) % 4) != 0)) {
    // Padded scale slots of the caller's output must read as zero scales.
    if (cudaMemsetAsync(sf, 0, static_cast<size_t>(qg_scale_bytes(rows, k, 16)), s) != cudaSuccess)
      return QG_ERR_CUDA;
  }
  // An error left pending by an earlier, unrelated call would be read back
  // below as this call's launch failure: report it without launching (and
  // without clearing it, so its owner still sees it).
  if (cudaPeekAtLastError() != cudaSuccess) return QG_ERR_CUDA;
  const int nparts = static_cast<int>((n + kChunk - 1) / kChunk);
  if (bf16) amax_partial_kernel<true><<<nparts, 256, 0, s>>>(x, n, scratch);
  else amax_partial_kernel<false><<<nparts, 256, 0, s>>>(x, n, scratch);
  amax_finalize_kernel<<<1, 1024, 0, s>>>(scratch, nparts);
  if (cudaGetLastError() != cudaSuccess ||
      launch_quantize_nvfp4(x, bf16, rows, k, layout, static_cast<uint8_t*>(q),
                            static_cast<uint8_t*>(sf), ts, scratch + kFinalSlot, s) != cudaSuccess) {
    forget_scratch_address();
    return QG_ERR_CUDA;
  }
  return QG_OK;
}

}  // extern "C"
