"""ctypes view of the CPU parity checker (TEST INFRASTRUCTURE ONLY).

Loads oracle/_build/libqg_oracle.so (this repo's restatement, qg_oracle.cpp)
and, when present, oracle/_ref/libqg_ref.so (the reference's own host headers
behind ref_shim.cpp).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs import this module.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libqg_oracle.so"
REF_SO = HERE / "_ref" / "libqg_ref.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
_I64, _I32, _U32, _U64, _F32, _U8 = (ctypes.c_int64, ctypes.c_int, ctypes.c_uint32,
                                     ctypes.c_uint64, ctypes.c_float, ctypes.c_uint8)
_fp = ctypes.POINTER(ctypes.c_float)

DISTRIBUTIONS = ["uniform", "normal", "laplace", "outlier", "lognormal", "constant"]


def build() -> None:
    """Compile the oracle (and the reference shim when a reference checkout exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load(path: Path) -> ctypes.CDLL:
    if not path.exists():
        build()
    return ctypes.CDLL(str(path))


class Oracle:
    def __init__(self) -> None:
        L = _load(ORACLE_SO)
        sig = {
            "qgo_encode_e2m1": (_U8, [_F32]),
            "qgo_decode_e2m1": (_F32, [_U8]),
            "qgo_decode_e4m3_positive": (_F32, [_U8]),
            "qgo_encode_e4m3_round_up": (_U8, [_F32]),
            "qgo_encode_e4m3_rn": (_U8, [_F32]),
            "qgo_decode_e4m3": (_F32, [_U8]),
            "qgo_decode_ue8m0": (_F32, [_U8]),
            "qgo_pack_e2m1x2": (_U8, [_U8, _U8]),
            "qgo_scale_offset": (_I64, [_I64, _I64, _I64, _I64, _I32, _I32]),
            "qgo_scale_storage_size": (_I64, [_I64, _I64, _I32]),
            "qgo_nvfp4_reference": (None, [_f32p, _I64, _u8p, _u8p, _fp]),
            "qgo_nvfp4_blocks_with_ts": (None, [_f32p, _I64, _F32, _u8p, _u8p]),
            "qgo_nvfp4_quantize_mma": (None, [_f32p, _I64, _I64, _I32, _u8p, _u8p, _fp]),
            "qgo_mxfp8_quantize": (None, [_f32p, _I64, _I64, _I32, _u8p, _u8p]),
            "qgo_block_scaled_gemm": (None, [_f32p, _f32p, _f32p, _f32p, _I64, _I64, _I64, _I32,
                                             _I64, _I64, _I32, _f32p]),
            "qgo_nvfp4_decode_mma": (None, [_u8p, _u8p, _I64, _I64, _I32, _f32p, _f32p]),
            "qgo_mxfp4_quantize": (None, [_f32p, _I64, _I64, _I32, _u8p, _u8p]),
            "qgo_mxfp4_decode": (None, [_u8p, _u8p, _I64, _I64, _I32, _f32p, _f32p]),
            "qgo_mxfp8_decode": (None, [_u8p, _u8p, _I64, _I64, _I32, _f32p, _f32p]),
            "qgo_fill_normal": (None, [_f32p, _I64, _U64, _F32, _F32]),
            "qgo_fill_requant_dist": (None, [_f32p, _I64, _U32, _I32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        self.L = L

    # -- inputs
    def normal(self, n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.L.qgo_fill_normal(out, n, seed, mean, std)
        return out

    def requant_dist(self, n: int, dist: str, seed: int = 1234) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.L.qgo_fill_requant_dist(out, n, seed, DISTRIBUTIONS.index(dist))
        return out

    # -- NVFP4
    def nvfp4_reference(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32).ravel()
        nb = (x.size + 15) // 16
        q = np.zeros(nb * 8, np.uint8)
        sf = np.zeros(nb, np.uint8)
        ts = ctypes.c_float(0)
        self.L.qgo_nvfp4_reference(x, x.size, q, sf, ctypes.byref(ts))
        return q, sf, ts.value

    def nvfp4_with_ts(self, x: np.ndarray, ts: float):
        """O1's block step under a given tensor scale (REF_LINEAR bytes)."""
        x = np.ascontiguousarray(x, np.float32).ravel()
        nb = (x.size + 15) // 16
        q = np.zeros(nb * 8, np.uint8)
        sf = np.zeros(nb, np.uint8)
        self.L.qgo_nvfp4_blocks_with_ts(x, x.size, float(ts), q, sf)
        return q, sf

    @staticmethod
    def linear_to_mma(q: np.ndarray, sf: np.ndarray, rows: int, k: int, order: int = 0):
        """REF_LINEAR NVFP4 bytes of a rows x k matrix -> MMA layout (low
        nibble first, scales at the L1 offsets of `order`; padded slots 0)."""
        q = np.ascontiguousarray(q, np.uint8)
        qm = ((q >> 4) | (q << 4)).astype(np.uint8)
        sfk = k // 16
        row_blocks, sf_blocks = (rows + 127) // 128, (sfk + 3) // 4
        r = np.repeat(np.arange(rows, dtype=np.int64), sfk)
        c = np.tile(np.arange(sfk, dtype=np.int64), rows)
        chunk = (c // 4) * row_blocks + r // 128 if order == 0 else (r // 128) * sf_blocks + c // 4
        w = r % 128
        off = chunk * 512 + (w % 32) * 16 + (w // 32) * 4 + c % 4
        out = np.zeros(row_blocks * sf_blocks * 512, np.uint8)
        out[off] = np.asarray(sf, np.uint8)[: rows * sfk]
        return qm, out

    def nvfp4_mma(self, x: np.ndarray, order: int = 0):
        rows, k = x.shape
        x = np.ascontiguousarray(x, np.float32)
        q = np.zeros(rows * k // 2, np.uint8)
        sf = np.zeros(self.L.qgo_scale_storage_size(rows, k, 16), np.uint8)
        ts = ctypes.c_float(0)
        self.L.qgo_nvfp4_quantize_mma(x, rows, k, order, q, sf, ctypes.byref(ts))
        return q, sf, ts.value

    def nvfp4_decode(self, q, sf, rows, k, order=0):
        v = np.empty(rows * k, np.float32)
        s = np.empty(rows * (k // 16), np.float32)
        self.L.qgo_nvfp4_decode_mma(np.ascontiguousarray(q), np.ascontiguousarray(sf), rows, k,
                                    order, v, s)
        return v, s

    # -- MXFP8
    def mxfp8(self, x: np.ndarray, order: int = 0):
        rows, k = x.shape
        x = np.ascontiguousarray(x, np.float32)
        q = np.zeros(rows * k, np.uint8)
        nsf = rows * (k // 32) if order < 0 else self.L.qgo_scale_storage_size(rows, k, 32)
        sf = np.zeros(nsf, np.uint8)
        self.L.qgo_mxfp8_quantize(x, rows, k, order, q, sf)
        return q, sf

    def mxfp4(self, x: np.ndarray, order: int = 0):
        rows, k = x.shape
        x = np.ascontiguousarray(x, np.float32)
        q = np.zeros(rows * k // 2, np.uint8)
        nsf = rows * (k // 32) if order < 0 else self.L.qgo_scale_storage_size(rows, k, 32)
        sf = np.zeros(nsf, np.uint8)
        self.L.qgo_mxfp4_quantize(x, rows, k, order, q, sf)
        return q, sf

    def mxfp4_decode(self, q, sf, rows, k, order=0):
        vals = np.zeros(rows * k, np.float32)
        scales = np.zeros(rows * (k // 32), np.float32)
        self.L.qgo_mxfp4_decode(np.ascontiguousarray(q), np.ascontiguousarray(sf), rows, k, order,
                                vals, scales)
        return vals, scales

    def mxfp8_decode(self, q, sf, rows, k, order=0):
        v = np.empty(rows * k, np.float32)
        s = np.empty(rows * (k // 32), np.float32)
        self.L.qgo_mxfp8_decode(np.ascontiguousarray(q), np.ascontiguousarray(sf), rows, k, order,
                                v, s)
        return v, s

    # -- selected rows of a large operand (sampled-row parity checks)
    @staticmethod
    def scale_rows(sf, rows_idx, nrows: int, k: int, sv: int, order: int = 0) -> np.ndarray:
        """Scale bytes [len(rows_idx), k/sv] of the given rows of an MMA-layout
        scale buffer (L1, scale_layout.hpp:11-26, in chunk order `order`)."""
        r = np.asarray(rows_idx, np.int64)[:, None]
        s = np.arange(k // sv, dtype=np.int64)[None, :]
        row_blocks, sf_blocks = (nrows + 127) // 128, (k // sv + 3) // 4
        chunk = (s // 4) * row_blocks + r // 128 if order == 0 else (r // 128) * sf_blocks + s // 4
        w = r % 128
        off = chunk * 512 + (w % 32) * 16 + (w // 32) * 4 + s % 4
        return np.asarray(sf, np.uint8)[off]

    def _luts(self):
        if not hasattr(self, "_lut"):
            self._lut = (np.array([self.L.qgo_decode_e2m1(i) for i in range(16)], np.float32),
                         np.array([self.L.qgo_decode_e4m3_positive(i) for i in range(256)], np.float32),
                         np.array([self.L.qgo_decode_e4m3(i) for i in range(256)], np.float32),
                         np.array([self.L.qgo_decode_ue8m0(i) for i in range(256)], np.float32))
        return self._lut

    def nvfp4_rows(self, q, sf, rows_idx, nrows: int, k: int, order: int = 0):
        """Logical (values [R*k], scales [R*k/16]) of the given rows of an
        MMA-layout NVFP4 operand (low nibble first), decoded with the same
        e2m1 / e4m3 tables as qgo_nvfp4_decode_mma."""
        e2m1, e4m3p, _, _ = self._luts()
        qb = np.asarray(q, np.uint8).reshape(nrows, k // 2)[np.asarray(rows_idx)]
        codes = np.stack([qb & 0xF, qb >> 4], axis=2).reshape(len(rows_idx), k)
        vals = e2m1[codes]
        scales = e4m3p[self.scale_rows(sf, rows_idx, nrows, k, 16, order)]
        return np.ascontiguousarray(vals.ravel()), np.ascontiguousarray(scales.ravel())

    def mxfp8_rows(self, q, sf, rows_idx, nrows: int, k: int, order: int = 0):
        """Logical (values, scales) of the given rows of an MMA-layout MXFP8
        operand (e4m3 bytes, ue8m0 per 32)."""
        _, _, e4m3, ue8m0 = self._luts()
        qb = np.asarray(q, np.uint8).reshape(nrows, k)[np.asarray(rows_idx)]
        scales = ue8m0[self.scale_rows(sf, rows_idx, nrows, k, 32, order)]
        return np.ascontiguousarray(e4m3[qb].ravel()), np.ascontiguousarray(scales.ravel())

    # -- O2
    def gemm(self, a, b, sfa, sfb, m, n, k, sv, rows=None, threads=8) -> np.ndarray:
        r0, r1 = (0, m) if rows is None else rows
        d = np.empty((r1 - r0) * n, np.float32)
        self.L.qgo_block_scaled_gemm(a, b, sfa, sfb, m, n, k, sv, r0, r1, threads, d)
        return d.reshape(r1 - r0, n)


class Reference:
    """The reference's own host oracles (built from its headers)."""

    def __init__(self) -> None:
        if not REF_SO.exists():
            build()
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} (needs the reference checkout to build)")
        L = ctypes.CDLL(str(REF_SO))
        sig = {
            "qgr_encode_e2m1": (_U8, [_F32]),
            "qgr_encode_e4m3_round_up": (_U8, [_F32]),
            "qgr_decode_e4m3_positive": (_F32, [_U8]),
            "qgr_nvfp4_reference": (None, [_f32p, _I64, _u8p, _u8p, _fp]),
            "qgr_scale_offset": (_I64, [_I32, _I32, _I32, _I32, _I32]),
            "qgr_scale_storage_size": (_I64, [_I32, _I32, _I32]),
            "qgr_block_scaled_gemm": (None, [_f32p, _f32p, _f32p, _f32p, _I32, _I32, _I32, _I32,
                                             _I32, _I32, _I32, _f32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        self.L = L

    def nvfp4_reference(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32).ravel()
        nb = (x.size + 15) // 16
        q = np.zeros(nb * 8, np.uint8)
        sf = np.zeros(nb, np.uint8)
        ts = ctypes.c_float(0)
        self.L.qgr_nvfp4_reference(x, x.size, q, sf, ctypes.byref(ts))
        return q, sf, ts.value

    def gemm(self, a, b, sfa, sfb, m, n, k, sv, rows=None, threads=1) -> np.ndarray:
        r0, r1 = (0, m) if rows is None else rows
        d = np.empty((r1 - r0) * n, np.float32)
        self.L.qgr_block_scaled_gemm(a, b, sfa, sfb, m, n, k, sv, r0, r1, threads, d)
        return d.reshape(r1 - r0, n)


def reference_available() -> bool:
    try:
        Reference()
        return True
    except (FileNotFoundError, OSError, subprocess.CalledProcessError):
        return False
