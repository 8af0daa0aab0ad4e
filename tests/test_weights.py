"""Quantised-weight files (cuda_optimazation_b200/weights.py): the .qgw
header and payload round trip on the host, malformed files are rejected, and
(GPU) loading into another layout equals quantising straight into it."""
import numpy as np
import pytest
import torch

from cuda_optimazation_b200 import qgemm, weights


def _nvfp4_host(oracle, rows, k, order=0):
    q, sf, ts = oracle.nvfp4_mma(oracle.normal(rows * k, 3).reshape(rows, k), order)
    return qgemm.Nvfp4Result(torch.from_numpy(q), torch.from_numpy(sf), torch.tensor([ts]),
                             rows, k, qgemm.LAYOUT_MMA if order == 0 else qgemm.LAYOUT_MMA_KMAJOR)


def test_roundtrip_nvfp4_and_mxfp4(oracle, tmp_path):
    r = _nvfp4_host(oracle, 130, 96)
    weights.save(tmp_path / "w.qgw", r)
    h = weights.read_header(tmp_path / "w.qgw")
    assert (h["format"], h["layout"], h["rows"], h["k"]) == (1, 1, 130, 96)
    assert np.float32(h["tensor_scale"]) == np.float32(r.tensor_scale.item())
    back = weights.load(tmp_path / "w.qgw", "cpu")
    assert torch.equal(back.quantized, r.quantized) and torch.equal(back.block_scales,
                                                                    r.block_scales)
    x = oracle.normal(64 * 128, 4).reshape(64, 128)
    q, sf = oracle.mxfp4(x, -1)
    m4 = qgemm.Mxfp4Result(torch.from_numpy(q), torch.from_numpy(sf), 64, 128,
                           qgemm.LAYOUT_REF_LINEAR)
    weights.save(tmp_path / "m.qgw", m4)
    back = weights.load(tmp_path / "m.qgw", "cpu")
    assert isinstance(back, qgemm.Mxfp4Result) and back.layout == qgemm.LAYOUT_REF_LINEAR
    assert torch.equal(back.quantized, m4.quantized)
    assert weights.main(["info", str(tmp_path / "m.qgw")]) == 0


def test_rejects_malformed(oracle, tmp_path):
    r = _nvfp4_host(oracle, 128, 64)
    p = tmp_path / "w.qgw"
    weights.save(p, r)
    raw = p.read_bytes()
    (tmp_path / "magic.qgw").write_bytes(b"XXXX" + raw[4:])
    (tmp_path / "short.qgw").write_bytes(raw[:-5])
    (tmp_path / "hdr.qgw").write_bytes(raw[:30])
    bad = bytearray(raw)
    bad[16] ^= 1  # rows no longer match the byte counts
    (tmp_path / "rows.qgw").write_bytes(bytes(bad))
    for name in ("magic", "short", "hdr", "rows"):
        with pytest.raises(ValueError):
            weights.load(tmp_path / f"{name}.qgw", "cpu")
    with pytest.raises(ValueError):  # layout changes need the GPU
        weights.load(p, "cpu", layout=qgemm.LAYOUT_REF_LINEAR)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4", "mxfp8"])
@pytest.mark.parametrize("shape", [(256, 512), (130, 96)])
def test_load_into_other_layouts(oracle, tmp_path, fmt, shape):
    rows, k = shape
    x = torch.from_numpy(oracle.normal(rows * k, 9).reshape(rows, k)).cuda()
    make = {"nvfp4": qgemm.make_nvfp4, "mxfp4": qgemm.make_mxfp4, "mxfp8": qgemm.make_mxfp8}[fmt]
    layouts = (qgemm.LAYOUT_REF_LINEAR, qgemm.LAYOUT_MMA, qgemm.LAYOUT_MMA_KMAJOR)
    direct = {lay: make(x, lay) for lay in layouts}
    for src in layouts:
        p = tmp_path / f"{fmt}_{src}.qgw"
        weights.save(p, direct[src])
        for dst in layouts:
            got = weights.load(p, "cuda", dst)
            torch.cuda.synchronize()
            assert got.layout == dst
            assert torch.equal(got.quantized, direct[dst].quantized), (src, dst)
            assert torch.equal(got.block_scales, direct[dst].block_scales), (src, dst)
