"""GPU parity: device quantizers vs the oracle, byte for byte."""
import numpy as np
import pytest
import torch

import oracle as om

pytestmark = pytest.mark.gpu

SHAPES = [(256, 256), (1024, 1024), (4096, 1024)]  # run_requant_epilogue_benchmark.sh


@pytest.mark.parametrize("dist", om.DISTRIBUTIONS)
@pytest.mark.parametrize("shape", SHAPES)
def test_nvfp4_ref_linear_bit_exact(qlib, oracle, dist, shape):
    rows, k = shape
    x = oracle.requant_dist(rows * k, dist, 1234)
    q, sf, ts = oracle.nvfp4_reference(x)
    r = qlib.make_nvfp4(torch.from_numpy(x.reshape(rows, k)).cuda(), qlib.LAYOUT_REF_LINEAR)
    torch.cuda.synchronize()
    assert float(r.tensor_scale.item()) == ts
    assert np.array_equal(r.quantized.cpu().numpy(), q), "values differ"
    assert np.array_equal(r.block_scales.cpu().numpy(), sf), "scales differ"


@pytest.mark.parametrize("layout,order", [(1, 0), (2, 1)])
@pytest.mark.parametrize("shape", [(256, 256), (130, 48), (384, 4096)])
def test_nvfp4_mma_layout_bit_exact(qlib, oracle, layout, order, shape):
    rows, k = shape
    x = oracle.normal(rows * k, 99 + rows).reshape(rows, k)
    q, sf, ts = oracle.nvfp4_mma(x, order)
    r = qlib.make_nvfp4(torch.from_numpy(x).cuda(), layout)
    torch.cuda.synchronize()
    assert float(r.tensor_scale.item()) == ts
    assert np.array_equal(r.quantized.cpu().numpy(), q)
    assert np.array_equal(r.block_scales.cpu().numpy(), sf)


def test_nvfp4_bf16_input_bit_exact(qlib, oracle):
    rows, k = 512, 1024
    x = torch.from_numpy(oracle.normal(rows * k, 5).reshape(rows, k)).to(torch.bfloat16)
    xf = x.float().numpy()  # exact widening
    q, sf, ts = oracle.nvfp4_mma(xf, 0)
    r = qlib.make_nvfp4(x.cuda(), qlib.LAYOUT_MMA)
    torch.cuda.synchronize()
    assert float(r.tensor_scale.item()) == ts
    assert np.array_equal(r.quantized.cpu().numpy(), q)
    assert np.array_equal(r.block_scales.cpu().numpy(), sf)


@pytest.mark.parametrize("n", [1, 15, 17, 1000, 4099])
def test_nvfp4_ragged_flat(qlib, oracle, n):
    x = oracle.requant_dist(n, "outlier", 3 + n)
    q, sf, ts = oracle.nvfp4_reference(x)
    r = qlib.make_nvfp4(torch.from_numpy(x.reshape(1, n)).cuda(), qlib.LAYOUT_REF_LINEAR)
    torch.cuda.synchronize()
    assert float(r.tensor_scale.item()) == ts
    assert np.array_equal(r.quantized.cpu().numpy(), q)
    assert np.array_equal(r.block_scales.cpu().numpy(), sf)


def test_nvfp4_zero_and_special(qlib, oracle):
    x = np.zeros((128, 64), np.float32)
    x[3, :16] = [0.0, -0.0, 1e-30, -1e-30, 5.0, -5.0, 2.5, 0.25, 0.75, 1.25, 1.75, 3.5, -3.5,
                 6.0, -6.0, 7.0]
    for arr in (x, np.zeros_like(x)):
        q, sf, ts = oracle.nvfp4_reference(arr)
        r = qlib.make_nvfp4(torch.from_numpy(arr).cuda(), qlib.LAYOUT_REF_LINEAR)
        torch.cuda.synchronize()
        assert float(r.tensor_scale.item()) == ts
        assert np.array_equal(r.quantized.cpu().numpy(), q)
        assert np.array_equal(r.block_scales.cpu().numpy(), sf)


def test_golden_fixtures_on_device(qlib):
    from pathlib import Path
    z = np.load(Path(__file__).resolve().parent / "golden" / "nvfp4_requant_64x64.npz")
    for dist in om.DISTRIBUTIONS:
        r = qlib.make_nvfp4(torch.from_numpy(z[f"{dist}_x"].reshape(64, 64)).cuda(),
                            qlib.LAYOUT_REF_LINEAR)
        torch.cuda.synchronize()
        assert np.array_equal(r.quantized.cpu().numpy(), z[f"{dist}_q"]), dist
        assert np.array_equal(r.block_scales.cpu().numpy(), z[f"{dist}_sf"]), dist
        assert np.float32(r.tensor_scale.item()) == z[f"{dist}_ts"][0], dist


@pytest.mark.parametrize("src,dst", [(0, 1), (1, 0), (1, 2), (2, 0)])
def test_repack_round_trip(qlib, oracle, src, dst):
    rows, k = 300, 512
    x = torch.from_numpy(oracle.normal(rows * k, 8).reshape(rows, k)).cuda()
    a = qlib.make_nvfp4(x, src)
    b = qlib.repack_nvfp4(a, dst)
    direct = qlib.make_nvfp4(x, dst)
    back = qlib.repack_nvfp4(b, src)
    torch.cuda.synchronize()
    assert torch.equal(b.quantized, direct.quantized)
    assert torch.equal(b.block_scales, direct.block_scales)
    assert torch.equal(back.quantized, a.quantized)
    assert torch.equal(back.block_scales, a.block_scales)


@pytest.mark.parametrize("layout,order", [(0, -1), (1, 0), (2, 1)])
@pytest.mark.parametrize("shape", [(256, 256), (200, 4096)])
def test_mxfp8_bit_exact(qlib, oracle, layout, order, shape):
    rows, k = shape
    x = oracle.normal(rows * k, 17).reshape(rows, k)
    x[0, :64] *= 1e-20  # tiny blocks
    x[1, :32] = 0.0     # all-zero block
    q, sf = oracle.mxfp8(x, order)
    r = qlib.make_mxfp8(torch.from_numpy(x).cuda(), layout)
    torch.cuda.synchronize()
    assert np.array_equal(r.quantized.cpu().numpy(), q)
    assert np.array_equal(r.block_scales.cpu().numpy(), sf)
