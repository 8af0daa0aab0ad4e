"""ctypes binding over the C ABI in include/qgemm.h, with torch-tensor wrappers.

The reference exposes its block-scaled path as C++ host routines
(``make_nvfp4_reference``, GEMMsm110/include/requant/nvfp4_reference.cuh:76-112;
``guide::block_scaled_reference_mnk``, cutlass-gemm-cpp-guide/include/guide/
block_scale_reference.hpp:10-37; ``guide::sm1xx_scale_offset`` /
``sm1xx_scale_storage_size``, scale_layout.hpp:11-34) and a CUTLASS GEMM binary.
This module offers the same operations on B200 device memory under the same
names: ``make_nvfp4`` returns an ``Nvfp4Result`` with ``quantized``,
``block_scales`` and ``tensor_scale`` fields like ``Nvfp4ReferenceResult``
(nvfp4_reference.cuh:18-22); ``block_scaled_gemm`` is the tensor-core GEMM over
those operands.

torch is used only for device memory and streams.  Every call goes to
libqgemm_b200.so; there is no fallback: a missing library raises.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libqgemm_b200.so"

# qg_status
OK, ERR_SHAPE, ERR_ALIGN, ERR_LAYOUT, ERR_DTYPE, ERR_CUDA, ERR_TIMEOUT, ERR_ARG, ERR_UNSUPPORTED = range(9)
# qg_dtype
DTYPE_F32, DTYPE_BF16 = 0, 1
# qg_layout
LAYOUT_REF_LINEAR, LAYOUT_MMA, LAYOUT_MMA_KMAJOR = 0, 1, 2
# qg_format
FORMAT_MXFP8, FORMAT_NVFP4, FORMAT_MXFP4 = 0, 1, 2

_VP, _I64, _I32, _U64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64

# name -> (restype, argtypes); mirrors include/qgemm.h one to one.
SIGNATURES = {
    "qg_status_string": (ctypes.c_char_p, [_I32]),
    "qg_version": (ctypes.c_char_p, []),
    "qg_scale_bytes": (_I64, [_I64, _I64, _I32]),
    "qg_quantize_workspace_bytes": (ctypes.c_size_t, []),
    "qg_quantize_nvfp4": (_I32, [_VP, _I32, _I64, _I64, _I32, _VP, _VP, _VP, _VP, _VP]),
    "qg_quantize_nvfp4_noalloc": (_I32, [_VP, _I32, _I64, _I64, _I32, _VP, _VP, _VP, _VP]),
    "qg_quantize_nvfp4_noalloc_max_elements": (_I64, []),
    "qg_quantize_mxfp8": (_I32, [_VP, _I32, _I64, _I64, _I32, _VP, _VP, _VP]),
    "qg_quantize_mxfp4": (_I32, [_VP, _I32, _I64, _I64, _I32, _VP, _VP, _VP]),
    "qg_gemm_mxfp4": (_I32, [_VP, _VP, _VP, _VP, _VP, _I32, _I64, _I64, _I64, _I64, _I32, _VP,
                             _VP]),
    "qg_repack_mx": (_I32, [_I32, _VP, _VP, _I32, _VP, _VP, _I32, _I64, _I64, _VP]),
    "qg_repack_nvfp4": (_I32, [_VP, _VP, _I32, _VP, _VP, _I32, _I64, _I64, _VP]),
    "qg_gemm_nvfp4": (_I32, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _I32, _I64, _I64, _I64, _I64,
                             _I32, _VP, _VP]),
    "qg_gemm_nvfp4_requant": (_I32, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I32, _VP,
                                     _I64, _I64, _I64, _I32, _VP, _VP]),
    "qg_gemm_mxfp8": (_I32, [_VP, _VP, _VP, _VP, _VP, _I32, _I64, _I64, _I64, _I64, _I32, _VP,
                             _VP]),
    "qg_gemm_nvfp4_skinny": (_I32, [_VP, _I32, _I64, _VP, _VP, _VP, _VP, _I32, _I64, _I64, _I64,
                                    _I32, _VP, ctypes.c_size_t, _VP, _VP]),
    "qg_gemm_nvfp4_skinny_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64]),
    "qg_gemm_nvfp4_gather": (_I32, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _I32, _I64, _I64, _I64,
                                    _I64, _I64, _I32, _VP, _VP]),
    "qg_ipc_export": (_I32, [_VP, _VP]),
    "qg_ipc_import": (_I32, [_VP, _VP]),
    "qg_ipc_close": (_I32, [_VP]),
    "qg_read_status": (_I32, [_VP, _VP, _VP]),
    "qg_plan_create_gemm": (_I32, [_VP, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I32, _I64,
                                   _I64, _I64, _I64, _I32, _VP]),
    "qg_plan_run": (_I32, [_VP, _VP]),
    "qg_plan_destroy": (_I32, [_VP]),
    "qg_selftest_e2m1_cvt": (_I32, [_VP, _VP]),
    "qg_selftest_wait_timeout": (_I32, [_U64, _VP, _VP]),
}

_lib: Optional[ctypes.CDLL] = None


class QGemmError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


def lib() -> ctypes.CDLL:
    """Load libqgemm_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m cuda_optimazation_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().qg_status_string(status).decode()


def _check(rc: int, what: str) -> None:
    if rc != OK:
        raise QGemmError(rc, what)


def _stream(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return DTYPE_F32
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    raise TypeError(f"unsupported input dtype {t.dtype}; use float32 or bfloat16")


def sm1xx_scale_storage_size(mn: int, k: int, sv: int) -> int:
    """Bytes of an MMA-layout scale buffer (scale_layout.hpp:28-34)."""
    return int(lib().qg_scale_bytes(mn, k, sv))


@dataclass
class Nvfp4Result:
    """Device twin of ``Nvfp4ReferenceResult`` (nvfp4_reference.cuh:18-22)."""
    quantized: torch.Tensor     # uint8, e2m1 pairs
    block_scales: torch.Tensor  # uint8, e4m3 per 16 K elements
    tensor_scale: torch.Tensor  # float32[1] on the device
    rows: int
    k: int
    layout: int


@dataclass
class Mxfp8Result:
    quantized: torch.Tensor     # uint8, e4m3
    block_scales: torch.Tensor  # uint8, ue8m0 per 32 K elements
    rows: int
    k: int
    layout: int


def make_nvfp4(x: torch.Tensor, layout: int = LAYOUT_MMA, workspace: Optional[torch.Tensor] = None,
               stream: Optional[torch.cuda.Stream] = None) -> Nvfp4Result:
    """Quantise a 2-D fp32/bf16 CUDA tensor to NVFP4 (bit-exact to
    make_nvfp4_reference over the same values)."""
    if x.dim() != 2 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D CUDA tensor")
    rows, k = x.shape
    n = rows * k
    nblocks = (n + 15) // 16
    dev = x.device
    q = torch.empty(nblocks * 8, dtype=torch.uint8, device=dev)
    if layout == LAYOUT_REF_LINEAR:
        sf = torch.empty(nblocks, dtype=torch.uint8, device=dev)
    else:
        sf = torch.empty(max(sm1xx_scale_storage_size(rows, k, 16), 1), dtype=torch.uint8, device=dev)
    ts = torch.empty(1, dtype=torch.float32, device=dev)
    if workspace is None:
        workspace = torch.empty(int(lib().qg_quantize_workspace_bytes()), dtype=torch.uint8, device=dev)
    rc = lib().qg_quantize_nvfp4(x.data_ptr(), _dtype_code(x), rows, k, layout, q.data_ptr(),
                                 sf.data_ptr(), ts.data_ptr(), workspace.data_ptr(), _stream(stream))
    _check(rc, "qg_quantize_nvfp4")
    return Nvfp4Result(q, sf, ts, rows, k, layout)


def make_mxfp8(x: torch.Tensor, layout: int = LAYOUT_MMA,
               stream: Optional[torch.cuda.Stream] = None) -> Mxfp8Result:
    """Quantise a 2-D fp32/bf16 CUDA tensor to MXFP8 (e4m3 + ue8m0 per 32)."""
    if x.dim() != 2 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D CUDA tensor")
    rows, k = x.shape
    q = torch.empty(rows * k, dtype=torch.uint8, device=x.device)
    nsf = rows * (k // 32) if layout == LAYOUT_REF_LINEAR else sm1xx_scale_storage_size(rows, k, 32)
    sf = torch.empty(max(nsf, 1), dtype=torch.uint8, device=x.device)
    rc = lib().qg_quantize_mxfp8(x.data_ptr(), _dtype_code(x), rows, k, layout, q.data_ptr(),
                                 sf.data_ptr(), _stream(stream))
    _check(rc, "qg_quantize_mxfp8")
    return Mxfp8Result(q, sf, rows, k, layout)


@dataclass
class Mxfp4Result:
    quantized: torch.Tensor     # uint8, e2m1 pairs
    block_scales: torch.Tensor  # uint8, ue8m0 per 32 K elements
    rows: int
    k: int
    layout: int


def make_mxfp4(x: torch.Tensor, layout: int = LAYOUT_MMA,
               stream: Optional[torch.cuda.Stream] = None) -> Mxfp4Result:
    """Quantise a 2-D fp32/bf16 CUDA tensor to MXFP4 (e2m1 + ue8m0 per 32)."""
    if x.dim() != 2 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous 2-D CUDA tensor")
    rows, k = x.shape
    q = torch.empty(rows * k // 2, dtype=torch.uint8, device=x.device)
    nsf = rows * (k // 32) if layout == LAYOUT_REF_LINEAR else sm1xx_scale_storage_size(rows, k, 32)
    sf = torch.empty(max(nsf, 1), dtype=torch.uint8, device=x.device)
    rc = lib().qg_quantize_mxfp4(x.data_ptr(), _dtype_code(x), rows, k, layout, q.data_ptr(),
                                 sf.data_ptr(), _stream(stream))
    _check(rc, "qg_quantize_mxfp4")
    return Mxfp4Result(q, sf, rows, k, layout)


def repack_nvfp4(src: Nvfp4Result, dst_layout: int,
                 stream: Optional[torch.cuda.Stream] = None) -> Nvfp4Result:
    """Re-lay NVFP4 values and scales (REF_LINEAR <-> MMA <-> MMA_KMAJOR)."""
    dev = src.quantized.device
    q = torch.empty_like(src.quantized)
    if dst_layout == LAYOUT_REF_LINEAR:
        sf = torch.empty(src.rows * src.k // 16, dtype=torch.uint8, device=dev)
    else:
        sf = torch.empty(sm1xx_scale_storage_size(src.rows, src.k, 16), dtype=torch.uint8, device=dev)
    rc = lib().qg_repack_nvfp4(src.quantized.data_ptr(), src.block_scales.data_ptr(), src.layout,
                               q.data_ptr(), sf.data_ptr(), dst_layout, src.rows, src.k,
                               _stream(stream))
    _check(rc, "qg_repack_nvfp4")
    return Nvfp4Result(q, sf, src.tensor_scale, src.rows, src.k, dst_layout)


def repack_mx(src, dst_layout: int, stream: Optional[torch.cuda.Stream] = None):
    """Re-lay an ``Mxfp4Result`` or ``Mxfp8Result`` (REF_LINEAR <-> MMA <->
    MMA_KMAJOR)."""
    dev = src.quantized.device
    bits = 4 if isinstance(src, Mxfp4Result) else 8
    q = torch.empty_like(src.quantized)
    nsf = (src.rows * (src.k // 32) if dst_layout == LAYOUT_REF_LINEAR
           else sm1xx_scale_storage_size(src.rows, src.k, 32))
    sf = torch.empty(nsf, dtype=torch.uint8, device=dev)
    rc = lib().qg_repack_mx(bits, src.quantized.data_ptr(), src.block_scales.data_ptr(),
                            src.layout, q.data_ptr(), sf.data_ptr(), dst_layout, src.rows, src.k,
                            _stream(stream))
    _check(rc, "qg_repack_mx")
    return type(src)(q, sf, src.rows, src.k, dst_layout)


def gemm_nvfp4_raw(a_q, a_sf, a_ts, b_q, b_sf, b_ts, c, m, n, k, sf_layout=LAYOUT_MMA,
                   status: Optional[torch.Tensor] = None, stream=None) -> None:
    """C = (a_ts*b_ts) * A . B^T into the preallocated tensor `c` (fp32 or bf16)."""
    rc = lib().qg_gemm_nvfp4(a_q.data_ptr(), a_sf.data_ptr(), _ptr(a_ts), b_q.data_ptr(),
                             b_sf.data_ptr(), _ptr(b_ts), c.data_ptr(), _dtype_code(c), m, n, k,
                             c.stride(0), sf_layout, _ptr(status), _stream(stream))
    _check(rc, "qg_gemm_nvfp4")


def gemm_mxfp8_raw(a_q, a_sf, b_q, b_sf, c, m, n, k, sf_layout=LAYOUT_MMA,
                   status: Optional[torch.Tensor] = None, stream=None) -> None:
    rc = lib().qg_gemm_mxfp8(a_q.data_ptr(), a_sf.data_ptr(), b_q.data_ptr(), b_sf.data_ptr(),
                             c.data_ptr(), _dtype_code(c), m, n, k, c.stride(0), sf_layout,
                             _ptr(status), _stream(stream))
    _check(rc, "qg_gemm_mxfp8")


def gemm_mxfp4_raw(a_q, a_sf, b_q, b_sf, c, m, n, k, sf_layout=LAYOUT_MMA,
                   status: Optional[torch.Tensor] = None, stream=None) -> None:
    rc = lib().qg_gemm_mxfp4(a_q.data_ptr(), a_sf.data_ptr(), b_q.data_ptr(), b_sf.data_ptr(),
                             c.data_ptr(), _dtype_code(c), m, n, k, c.stride(0), sf_layout,
                             _ptr(status), _stream(stream))
    _check(rc, "qg_gemm_mxfp4")


def block_scaled_gemm(a, b, out_dtype: torch.dtype = torch.bfloat16,
                      out: Optional[torch.Tensor] = None,
                      status: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Tensor-core GEMM C = A . B^T over two quantised operands of the same
    format (``Nvfp4Result``, ``Mxfp8Result`` or ``Mxfp4Result`` pair, both in
    one MMA layout)."""
    if type(a) is not type(b):
        raise ValueError("operands must share the format")
    if a.k != b.k or a.layout != b.layout:
        raise ValueError("operands must share K and layout")
    m, n, k = a.rows, b.rows, a.k
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, device=a.quantized.device)
    if isinstance(a, Nvfp4Result):
        gemm_nvfp4_raw(a.quantized, a.block_scales, a.tensor_scale, b.quantized, b.block_scales,
                       b.tensor_scale, out, m, n, k, a.layout, status, stream)
    elif isinstance(a, Mxfp4Result):
        gemm_mxfp4_raw(a.quantized, a.block_scales, b.quantized, b.block_scales, out, m, n, k,
                       a.layout, status, stream)
    else:
        gemm_mxfp8_raw(a.quantized, a.block_scales, b.quantized, b.block_scales, out, m, n, k,
                       a.layout, status, stream)
    return out


def gemm_nvfp4_requant_raw(a_q, a_sf, a_ts, b_q, b_sf, b_ts, out_ts, out_q, out_sf, m, n, k,
                           out_layout=LAYOUT_REF_LINEAR, sf_layout=LAYOUT_MMA,
                           out_amax: Optional[torch.Tensor] = None,
                           status: Optional[torch.Tensor] = None, stream=None) -> None:
    """NVFP4 output of A . B^T into preallocated uint8 tensors out_q (m*n/2
    bytes) and out_sf (m*n/16 bytes, or the MMA layout's size)."""
    rc = lib().qg_gemm_nvfp4_requant(a_q.data_ptr(), a_sf.data_ptr(), _ptr(a_ts), b_q.data_ptr(),
                                     b_sf.data_ptr(), _ptr(b_ts), _ptr(out_ts), out_q.data_ptr(),
                                     out_sf.data_ptr(), out_layout, _ptr(out_amax), m, n, k,
                                     sf_layout, _ptr(status), _stream(stream))
    _check(rc, "qg_gemm_nvfp4_requant")


def gemm_nvfp4_requant(a: Nvfp4Result, b: Nvfp4Result, out_ts: torch.Tensor,
                       out_layout: int = LAYOUT_REF_LINEAR,
                       out_amax: Optional[torch.Tensor] = None,
                       status: Optional[torch.Tensor] = None, stream=None) -> Nvfp4Result:
    """NVFP4 GEMM whose output is requantised to NVFP4 in the epilogue (the
    tc6 fused epilogue, GEMMsm110/include/backends/tc6_nvfp4.cuh:460-503).
    ``out_ts`` is the output's tensor scale (float32[1] on the device), given
    by the caller as tc6 takes its inverse; the result is an ``Nvfp4Result``
    of m rows and n columns in ``out_layout``.  ``out_amax`` (int32[1] on the
    device, zeroed by the caller) receives the float bit pattern of the
    output's amax."""
    if a.k != b.k or a.layout != b.layout:
        raise ValueError("operands must share K and layout")
    m, n, k = a.rows, b.rows, a.k
    dev = a.quantized.device
    q = torch.empty(m * n // 2, dtype=torch.uint8, device=dev)
    if out_layout == LAYOUT_REF_LINEAR:
        sf = torch.empty(m * n // 16, dtype=torch.uint8, device=dev)
    else:
        sf = torch.empty(sm1xx_scale_storage_size(m, n, 16), dtype=torch.uint8, device=dev)
    gemm_nvfp4_requant_raw(a.quantized, a.block_scales, a.tensor_scale, b.quantized,
                           b.block_scales, b.tensor_scale, out_ts, q, sf, m, n, k, out_layout,
                           a.layout, out_amax, status, stream)
    return Nvfp4Result(q, sf, out_ts, m, n, out_layout)


class GemmPlan:
    """A ``qg_plan``: one GEMM call C = A . B^T bound to fixed buffers, its
    host work (checks, tensor-map encodes, kernel choice) done once;
    ``run()`` only enqueues the kernel and reads the operands' current
    contents.  The tensors are kept alive by the plan."""

    def __init__(self, a, b, out: torch.Tensor, status: Optional[torch.Tensor] = None):
        if type(a) is not type(b) or a.k != b.k or a.layout != b.layout:
            raise ValueError("operands must share format, K and layout")
        fmt = {Nvfp4Result: FORMAT_NVFP4, Mxfp8Result: FORMAT_MXFP8,
               Mxfp4Result: FORMAT_MXFP4}[type(a)]
        ats = a.tensor_scale if fmt == FORMAT_NVFP4 else None
        bts = b.tensor_scale if fmt == FORMAT_NVFP4 else None
        self._keep = (a, b, out, status)
        self._h = ctypes.c_void_p()
        rc = lib().qg_plan_create_gemm(ctypes.byref(self._h), fmt, a.quantized.data_ptr(),
                                       a.block_scales.data_ptr(), _ptr(ats), b.quantized.data_ptr(),
                                       b.block_scales.data_ptr(), _ptr(bts), out.data_ptr(),
                                       _dtype_code(out), a.rows, b.rows, a.k, out.stride(0),
                                       a.layout, _ptr(status))
        _check(rc, "qg_plan_create_gemm")
        self.out = out

    def run(self, stream=None) -> torch.Tensor:
        if not self._h:
            raise RuntimeError("plan is closed")
        _check(lib().qg_plan_run(self._h, _stream(stream)), "qg_plan_run")
        return self.out

    def close(self) -> None:
        if self._h:
            lib().qg_plan_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def skinny_workspace(m: int, n: int, k: int, device) -> torch.Tensor:
    """A workspace for gemm_nvfp4_skinny (reusable across calls on one
    stream; every call rewrites the state it reads, so no zero fill is
    needed -- it is zero-filled here only to make it deterministic)."""
    need = int(lib().qg_gemm_nvfp4_skinny_workspace_bytes(m, n, k))
    return torch.zeros(need, dtype=torch.uint8, device=device)


def gemm_nvfp4_skinny(x: torch.Tensor, w: "Nvfp4Result", out_dtype: torch.dtype = torch.bfloat16,
                      out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                      status: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Decode GEMM C = x . w^T with the activation quantisation fused in:
    x is an (m <= 128) x k fp32/bf16 CUDA tensor, w pre-quantised NVFP4
    weights (n x k, MMA layout)."""
    m, k = x.shape
    n = w.rows
    if w.k != k:
        raise ValueError("K mismatch")
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, device=x.device)
    need = int(lib().qg_gemm_nvfp4_skinny_workspace_bytes(m, n, k))
    if workspace is None or workspace.numel() < need:
        workspace = skinny_workspace(m, n, k, x.device)
    rc = lib().qg_gemm_nvfp4_skinny(x.data_ptr(), _dtype_code(x), m, w.quantized.data_ptr(),
                                    w.block_scales.data_ptr(), w.tensor_scale.data_ptr(),
                                    out.data_ptr(), _dtype_code(out), n, k, out.stride(0),
                                    w.layout, workspace.data_ptr(), workspace.numel(),
                                    _ptr(status), _stream(stream))
    _check(rc, "qg_gemm_nvfp4_skinny")
    return out


IPC_HANDLE_BYTES = 72
MAX_RANKS = 8


def ipc_export(t: torch.Tensor) -> bytes:
    """CUDA IPC handle (+ offset) of the device buffer behind `t`."""
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib().qg_ipc_export(t.data_ptr(), buf), "qg_ipc_export")
    return buf.raw


def ipc_import(handle: bytes) -> int:
    """Map a peer's buffer (from ipc_export in another process); returns the
    device pointer in this process."""
    ptr = ctypes.c_void_p()
    _check(lib().qg_ipc_import(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES),
                               ctypes.byref(ptr)), "qg_ipc_import")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    _check(lib().qg_ipc_close(ctypes.c_void_p(ptr)), "qg_ipc_close")


def gemm_nvfp4_gather(a: "Nvfp4Result", b_local: "Nvfp4Result", c_ptrs: list[int], col0: int,
                      ldc: int, status: Optional[torch.Tensor] = None, stream=None) -> None:
    """Column-parallel GEMM with the all-gather fused in: computes
    C[:, col0:col0+b_local.rows] = A . B_local^T (bf16) into every buffer of
    c_ptrs (this rank's own full C and the peers' IPC-mapped ones)."""
    if len(c_ptrs) < 1 or len(c_ptrs) > MAX_RANKS:
        raise ValueError("1..8 output buffers")
    arr = (ctypes.c_void_p * len(c_ptrs))(*c_ptrs)
    rc = lib().qg_gemm_nvfp4_gather(a.quantized.data_ptr(), a.block_scales.data_ptr(),
                                    a.tensor_scale.data_ptr(), b_local.quantized.data_ptr(),
                                    b_local.block_scales.data_ptr(),
                                    b_local.tensor_scale.data_ptr(), arr, len(c_ptrs), col0,
                                    a.rows, b_local.rows, a.k, ldc, a.layout, _ptr(status),
                                    _stream(stream))
    _check(rc, "qg_gemm_nvfp4_gather")


def read_status(status: torch.Tensor, stream=None) -> tuple[int, int]:
    """(qg_status, raw device code) of a status word; clears it."""
    code = ctypes.c_uint32(0)
    rc = lib().qg_read_status(status.data_ptr(), ctypes.addressof(code), _stream(stream))
    return rc, code.value


def selftest_wait_timeout(timeout_ns: int, status: torch.Tensor, stream=None) -> None:
    _check(lib().qg_selftest_wait_timeout(timeout_ns, status.data_ptr(), _stream(stream)),
           "qg_selftest_wait_timeout")
