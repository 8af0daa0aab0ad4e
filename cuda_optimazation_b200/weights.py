"""Quantised-weight files: store NVFP4 / MXFP4 / MXFP8 operands once and load
them without re-quantising (the decode GEMM's pre-quantised weights).

The reference keeps a quantised tensor only in memory, as
``Nvfp4ReferenceResult`` (values, block scales, tensor scale;
GEMMsm110/include/requant/nvfp4_reference.cuh:18-22).  A ``.qgw`` file holds
the same three parts plus the format and the layout tag, so a file written in
the reference's byte order (QG_LAYOUT_REF_LINEAR) can be loaded straight into
the tensor-core layout and vice versa.  Layout changes run on the GPU
(qg_repack_nvfp4 / qg_repack_mx); the file itself is plain bytes.

File layout (little-endian):

    offset  size  field
    0       4     magic b"QGW1"
    4       4     version (1)
    8       4     format: 0 MXFP8, 1 NVFP4, 2 MXFP4
    12      4     layout: 0 REF_LINEAR, 1 MMA, 2 MMA_KMAJOR
    16      8     rows
    24      8     k (elements per row)
    32      4     tensor scale (fp32; 1.0 for the MX formats)
    36      4     reserved (0)
    40      8     value bytes V
    48      8     scale bytes S
    56      8     reserved (0)
    64      V     values
    64+V    S     scales

Command line::

    python -m cuda_optimazation_b200.weights info FILE
    python -m cuda_optimazation_b200.weights repack IN OUT --layout mma|kmajor|linear
"""
from __future__ import annotations

import argparse
import struct
import sys
from pathlib import Path
from typing import Optional, Union

import torch

from . import qgemm

MAGIC = b"QGW1"
VERSION = 1
FMT_MXFP8, FMT_NVFP4, FMT_MXFP4 = 0, 1, 2
_HEADER = struct.Struct("<4sIIIqqfIqqq")
HEADER_BYTES = 64
assert _HEADER.size == HEADER_BYTES

Result = Union[qgemm.Nvfp4Result, qgemm.Mxfp4Result, qgemm.Mxfp8Result]
_LAYOUT_NAMES = {"linear": qgemm.LAYOUT_REF_LINEAR, "mma": qgemm.LAYOUT_MMA,
                 "kmajor": qgemm.LAYOUT_MMA_KMAJOR}


def _fmt_of(r: Result) -> int:
    if isinstance(r, qgemm.Nvfp4Result):
        return FMT_NVFP4
    if isinstance(r, qgemm.Mxfp4Result):
        return FMT_MXFP4
    if isinstance(r, qgemm.Mxfp8Result):
        return FMT_MXFP8
    raise TypeError(f"not a quantised operand: {type(r).__name__}")


def expected_bytes(fmt: int, layout: int, rows: int, k: int) -> tuple[int, int]:
    """(value bytes, scale bytes) of a rows x k operand."""
    sv = 16 if fmt == FMT_NVFP4 else 32
    vbytes = rows * k // 2 if fmt in (FMT_NVFP4, FMT_MXFP4) else rows * k
    if layout == qgemm.LAYOUT_REF_LINEAR:
        sbytes = rows * k // sv
    else:
        sbytes = qgemm.sm1xx_scale_storage_size(rows, k, sv)
    return vbytes, sbytes


def save(path: Union[str, Path], r: Result) -> None:
    """Write a quantised operand (device or host tensors) to ``path``."""
    fmt = _fmt_of(r)
    ts = 1.0
    if fmt == FMT_NVFP4 and r.tensor_scale is not None:
        ts = float(r.tensor_scale.reshape(-1)[0].item())
    q = r.quantized.detach().reshape(-1).to("cpu", torch.uint8)
    sf = r.block_scales.detach().reshape(-1).to("cpu", torch.uint8)
    vb, sb = expected_bytes(fmt, r.layout, r.rows, r.k)
    if q.numel() < vb or sf.numel() < sb:
        raise ValueError("operand buffers are smaller than its shape needs")
    header = _HEADER.pack(MAGIC, VERSION, fmt, r.layout, r.rows, r.k, ts, 0, vb, sb, 0)
    with open(path, "wb") as f:
        f.write(header)
        f.write(q[:vb].numpy().tobytes())
        f.write(sf[:sb].numpy().tobytes())


def read_header(path: Union[str, Path]) -> dict:
    with open(path, "rb") as f:
        raw = f.read(HEADER_BYTES)
    if len(raw) != HEADER_BYTES:
        raise ValueError(f"{path}: truncated header")
    magic, ver, fmt, layout, rows, k, ts, _, vb, sb, _ = _HEADER.unpack(raw)
    if magic != MAGIC:
        raise ValueError(f"{path}: not a QGW file")
    if ver != VERSION:
        raise ValueError(f"{path}: unsupported version {ver}")
    if fmt not in (FMT_MXFP8, FMT_NVFP4, FMT_MXFP4) or layout not in (0, 1, 2):
        raise ValueError(f"{path}: bad format / layout tag")
    if (vb, sb) != expected_bytes(fmt, layout, rows, k):
        raise ValueError(f"{path}: byte counts do not match the shape")
    return dict(format=fmt, layout=layout, rows=rows, k=k, tensor_scale=ts, value_bytes=vb,
                scale_bytes=sb)


def load(path: Union[str, Path], device: Union[str, torch.device] = "cuda",
         layout: Optional[int] = None, stream=None) -> Result:
    """Read a ``.qgw`` file onto ``device``; ``layout`` (optional) re-lays it
    on the GPU (only a CUDA device can change the layout)."""
    h = read_header(path)
    with open(path, "rb") as f:
        f.seek(HEADER_BYTES)
        q = torch.frombuffer(bytearray(f.read(h["value_bytes"])), dtype=torch.uint8)
        sf = torch.frombuffer(bytearray(f.read(h["scale_bytes"])), dtype=torch.uint8)
    if q.numel() != h["value_bytes"] or sf.numel() != h["scale_bytes"]:
        raise ValueError(f"{path}: truncated payload")
    device = torch.device(device)
    q, sf = q.to(device), sf.to(device)
    fmt, rows, k, lay = h["format"], h["rows"], h["k"], h["layout"]
    if fmt == FMT_NVFP4:
        ts = torch.tensor([h["tensor_scale"]], dtype=torch.float32, device=device)
        r: Result = qgemm.Nvfp4Result(q, sf, ts, rows, k, lay)
    elif fmt == FMT_MXFP4:
        r = qgemm.Mxfp4Result(q, sf, rows, k, lay)
    else:
        r = qgemm.Mxfp8Result(q, sf, rows, k, lay)
    if layout is not None and layout != lay:
        if device.type != "cuda":
            raise ValueError("layout changes run on the GPU: load onto a CUDA device")
        r = repack(r, layout, stream)
    return r


def repack(r: Result, layout: int, stream=None) -> Result:
    """Re-lay a device operand (qg_repack_nvfp4 / qg_repack_mx)."""
    if isinstance(r, qgemm.Nvfp4Result):
        return qgemm.repack_nvfp4(r, layout, stream)
    return qgemm.repack_mx(r, layout, stream)


def main(argv: Optional[list[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m cuda_optimazation_b200.weights")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p_info = sub.add_parser("info", help="print a file's header")
    p_info.add_argument("file")
    p_rep = sub.add_parser("repack", help="re-lay a file (on the GPU)")
    p_rep.add_argument("src")
    p_rep.add_argument("dst")
    p_rep.add_argument("--layout", choices=sorted(_LAYOUT_NAMES), required=True)
    args = ap.parse_args(argv)
    if args.cmd == "info":
        h = read_header(args.file)
        names = {FMT_MXFP8: "mxfp8", FMT_NVFP4: "nvfp4", FMT_MXFP4: "mxfp4"}
        lnames = {v: k for k, v in _LAYOUT_NAMES.items()}
        print(f"format={names[h['format']]} layout={lnames[h['layout']]} rows={h['rows']} "
              f"k={h['k']} tensor_scale={h['tensor_scale']:.9g} value_bytes={h['value_bytes']} "
              f"scale_bytes={h['scale_bytes']}")
        return 0
    r = load(args.src, "cuda", _LAYOUT_NAMES[args.layout])
    save(args.dst, r)
    return 0


if __name__ == "__main__":
    sys.exit(main())
