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
