"""CPU checks of the C ABI: the library loads, exports every symbol the
header declares, and rejects bad arguments before touching the GPU."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_symbols():
    text = (ROOT / "include" / "qgemm.h").read_text()
    return sorted(set(re.findall(r"\b(qg_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported(qlib):
    import ctypes
    handle = ctypes.CDLL(str(qlib.LIB_PATH))
    syms = header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(handle, s), s
    assert set(syms) == set(qlib.SIGNATURES), "python signatures must mirror the header"


def test_scale_bytes(qlib):
    L = qlib.lib()
    assert L.qg_scale_bytes(128, 128, 32) == 512
    assert L.qg_scale_bytes(129, 129, 32) == 2048
    assert L.qg_scale_bytes(8192, 8192, 16) == 64 * 128 * 512
    assert L.qg_scale_bytes(-1, 4, 16) == -1


def test_status_strings(qlib):
    for code in range(9):
        assert qlib.status_string(code)
    assert qlib.status_string(0) == "ok"


def test_argument_validation_without_gpu(qlib):
    L = qlib.lib()
    # Null operands are rejected before any CUDA call.
    assert L.qg_gemm_nvfp4(None, None, None, None, None, None, None, 1, 256, 256, 256, 256, 1,
                           None, None) == qlib.ERR_ARG
    assert L.qg_quantize_nvfp4(None, 0, 1, 16, 1, None, None, None, None, None) == qlib.ERR_ARG
    assert L.qg_read_status(None, None, None) == qlib.ERR_ARG


def test_gather_and_ipc_argument_validation_without_gpu(qlib):
    import ctypes
    L = qlib.lib()
    one = (ctypes.c_void_p * 1)(ctypes.c_void_p(16))
    nine = (ctypes.c_void_p * 9)(*([ctypes.c_void_p(16)] * 9))
    # Rank count outside 1..8 and a shard that runs past ldc are rejected first.
    assert L.qg_gemm_nvfp4_gather(None, None, None, None, None, None, one, 0, 0, 256, 256, 256,
                                  256, 1, None, None) == qlib.ERR_ARG
    assert L.qg_gemm_nvfp4_gather(None, None, None, None, None, None, nine, 9, 0, 256, 256, 256,
                                  256, 1, None, None) == qlib.ERR_ARG
    assert L.qg_gemm_nvfp4_gather(None, None, None, None, None, None, one, 1, 128, 256, 256, 256,
                                  256, 1, None, None) == qlib.ERR_SHAPE
    assert L.qg_gemm_nvfp4_gather(None, None, None, None, None, None, None, 1, 0, 256, 256, 256,
                                  256, 1, None, None) == qlib.ERR_ARG
    assert L.qg_ipc_export(None, None) == qlib.ERR_ARG
    assert L.qg_ipc_import(None, None) == qlib.ERR_ARG
    assert L.qg_ipc_close(ctypes.c_void_p(4096)) == qlib.ERR_ARG  # never imported
    assert qlib.IPC_HANDLE_BYTES == 72 and qlib.MAX_RANKS == 8


def test_new_entry_points_validate_without_gpu(qlib):
    """MXFP4 quantizer / GEMM, MX repack, NVFP4-output GEMM and the e2m1
    self test reject bad arguments before any CUDA call (fake, aligned
    addresses are never dereferenced)."""
    L = qlib.lib()
    a, mis = 4096, 4104  # 16-byte aligned / misaligned fake device addresses
    # qg_quantize_mxfp4(x, dtype, rows, k, layout, q, sf, stream)
    assert L.qg_quantize_mxfp4(None, 0, 1, 32, 1, a, a, None) == qlib.ERR_ARG
    assert L.qg_quantize_mxfp4(a, 9, 1, 32, 1, a, a, None) == qlib.ERR_DTYPE
    assert L.qg_quantize_mxfp4(a, 0, 1, 32, 5, a, a, None) == qlib.ERR_LAYOUT
    assert L.qg_quantize_mxfp4(a, 0, 1, 48, 1, a, a, None) == qlib.ERR_SHAPE
    assert L.qg_quantize_mxfp4(mis, 0, 1, 32, 1, a, a, None) == qlib.ERR_ALIGN
    # qg_gemm_mxfp4(a_q, a_sf, b_q, b_sf, c, c_dtype, m, n, k, ldc, sf_layout, status, stream)
    assert L.qg_gemm_mxfp4(None, a, a, a, a, 1, 256, 256, 256, 256, 1, None, None) == qlib.ERR_ARG
    assert L.qg_gemm_mxfp4(a, a, a, a, a, 3, 256, 256, 256, 256, 1, None, None) == qlib.ERR_DTYPE
    assert L.qg_gemm_mxfp4(a, a, a, a, a, 1, 256, 256, 256, 256, 0, None, None) == qlib.ERR_LAYOUT
    assert L.qg_gemm_mxfp4(a, a, a, a, a, 1, 256, 256, 48, 256, 1, None, None) == qlib.ERR_SHAPE
    assert L.qg_gemm_mxfp4(mis, a, a, a, a, 1, 256, 256, 256, 256, 1, None, None) == qlib.ERR_ALIGN
    # qg_repack_mx(bits, src_q, src_sf, src_layout, dst_q, dst_sf, dst_layout, rows, k, stream)
    assert L.qg_repack_mx(4, None, a, 0, a, a, 1, 128, 64, None) == qlib.ERR_ARG
    assert L.qg_repack_mx(6, a, a, 0, a, a, 1, 128, 64, None) == qlib.ERR_DTYPE
    assert L.qg_repack_mx(4, a, a, 3, a, a, 1, 128, 64, None) == qlib.ERR_LAYOUT
    assert L.qg_repack_mx(8, a, a, 0, a, a, 1, 128, 48, None) == qlib.ERR_SHAPE
    assert L.qg_repack_mx(4, mis, a, 0, a, a, 1, 128, 64, None) == qlib.ERR_ALIGN
    # qg_gemm_nvfp4_requant(..., out_ts, out_q, out_sf, out_layout, out_amax, m, n, k, ...)
    assert L.qg_gemm_nvfp4_requant(a, a, None, a, a, None, None, None, a, 0, None, 128, 128, 128,
                                   1, None, None) == qlib.ERR_ARG
    assert L.qg_gemm_nvfp4_requant(a, a, None, a, a, None, None, a, a, 4, None, 128, 128, 128,
                                   1, None, None) == qlib.ERR_LAYOUT
    assert L.qg_gemm_nvfp4_requant(a, a, None, a, a, None, None, a, a, 0, None, 128, 40, 128,
                                   1, None, None) == qlib.ERR_SHAPE
    assert L.qg_gemm_nvfp4_requant(a, a, None, a, a, None, None, mis, a, 0, None, 128, 128, 128,
                                   1, None, None) == qlib.ERR_ALIGN
    assert L.qg_selftest_e2m1_cvt(None, None) == qlib.ERR_ARG


def test_plan_argument_validation_without_gpu(qlib):
    import ctypes
    L = qlib.lib()
    h = ctypes.c_void_p()
    a = 4096
    assert L.qg_plan_create_gemm(None, 1, a, a, None, a, a, None, a, 1, 256, 256, 256, 256, 1,
                                 None) == qlib.ERR_ARG
    assert L.qg_plan_create_gemm(ctypes.byref(h), 7, a, a, None, a, a, None, a, 1, 256, 256, 256,
                                 256, 1, None) == qlib.ERR_DTYPE
    assert L.qg_plan_create_gemm(ctypes.byref(h), 1, None, a, None, a, a, None, a, 1, 256, 256,
                                 256, 256, 1, None) == qlib.ERR_ARG
    assert L.qg_plan_create_gemm(ctypes.byref(h), 0, a, a, None, a, a, None, a, 1, 256, 256, 48,
                                 256, 1, None) == qlib.ERR_SHAPE
    assert not h.value  # no plan on failure
    assert L.qg_plan_run(None, None) == qlib.ERR_ARG
    assert L.qg_plan_destroy(None) == qlib.ERR_ARG
