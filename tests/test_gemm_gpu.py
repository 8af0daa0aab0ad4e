"""GPU parity: tcgen05 block-scaled GEMMs vs the oracle's O2
(block_scaled_reference_mnk, double accumulation) within the stated
tolerance (tests/helpers.py)."""
import numpy as np
import pytest
import torch

from helpers import check_gemm

pytestmark = pytest.mark.gpu


def nvfp4_case(oracle, qlib, m, n, k, layout=1, seed=20260817, b_std=1.0):
    xa = oracle.normal(m * k, seed).reshape(m, k)
    xb = oracle.normal(n * k, seed ^ 0xBB67AE85, 0.0, b_std).reshape(n, k)
    order = 0 if layout == 1 else 1
    qa, sa, ta = oracle.nvfp4_mma(xa, order)
    qb, sb, tb = oracle.nvfp4_mma(xb, order)
    return (qa, sa, ta), (qb, sb, tb), order


def oracle_nvfp4(oracle, a, b, m, n, k, order, rows=None):
    av, asf = oracle.nvfp4_decode(a[0], a[1], m, k, order)
    bv, bsf = oracle.nvfp4_decode(b[0], b[1], n, k, order)
    d = oracle.gemm(av, bv, asf, bsf, m, n, k, 16, rows=rows)
    return d * np.float32(np.float32(a[2]) * np.float32(b[2]))


def run_nvfp4(qlib, a, b, m, n, k, layout, out_dtype):
    dev = torch.device("cuda")
    t = lambda arr: torch.from_numpy(arr).to(dev)
    ats = torch.tensor([a[2]], dtype=torch.float32, device=dev)
    bts = torch.tensor([b[2]], dtype=torch.float32, device=dev)
    c = torch.full((m, n), float("nan"), dtype=out_dtype, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    qlib.gemm_nvfp4_raw(t(a[0]), t(a[1]), ats, t(b[0]), t(b[1]), bts, c, m, n, k, layout, status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, f"device status {code}"
    return c.float().cpu().numpy()


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (256, 256, 256), (256, 512, 1024)])
def test_nvfp4_fp32(qlib, oracle, m, n, k):
    a, b, order = nvfp4_case(oracle, qlib, m, n, k)
    got = run_nvfp4(qlib, a, b, m, n, k, 1, torch.float32)
    check_gemm(got, oracle_nvfp4(oracle, a, b, m, n, k, order))


def test_nvfp4_bf16_256(qlib, oracle):
    m = n = k = 256
    a, b, order = nvfp4_case(oracle, qlib, m, n, k)
    got = run_nvfp4(qlib, a, b, m, n, k, 1, torch.bfloat16)
    check_gemm(got, oracle_nvfp4(oracle, a, b, m, n, k, order), bf16=True)


@pytest.mark.parametrize("m,n,k", [(130, 129, 128), (1, 300, 96), (333, 17, 544), (64, 1000, 32)])
def test_nvfp4_ragged(qlib, oracle, m, n, k):
    a, b, order = nvfp4_case(oracle, qlib, m, n, k)
    got = run_nvfp4(qlib, a, b, m, n, k, 1, torch.float32)
    check_gemm(got, oracle_nvfp4(oracle, a, b, m, n, k, order))


def test_nvfp4_kmajor_scale_order(qlib, oracle):
    m, n, k = 384, 512, 1536
    a, b, order = nvfp4_case(oracle, qlib, m, n, k, layout=2)
    got = run_nvfp4(qlib, a, b, m, n, k, 2, torch.float32)
    check_gemm(got, oracle_nvfp4(oracle, a, b, m, n, k, order))


def test_nvfp4_1024_sampled_rows(qlib, oracle):
    m = n = k = 1024
    a, b, order = nvfp4_case(oracle, qlib, m, n, k)
    got = run_nvfp4(qlib, a, b, m, n, k, 1, torch.float32)
    rows = (512, 640)
    check_gemm(got[rows[0]:rows[1]], oracle_nvfp4(oracle, a, b, m, n, k, order, rows=rows))


def mxfp8_case(oracle, m, n, k, layout=1):
    order = 0 if layout == 1 else 1
    xa = oracle.normal(m * k, 11).reshape(m, k)
    xb = oracle.normal(n * k, 12, 0.0, 0.02).reshape(n, k)
    return oracle.mxfp8(xa, order), oracle.mxfp8(xb, order), order


@pytest.mark.parametrize("m,n,k,out", [(256, 256, 256, torch.float32), (130, 300, 544, torch.float32),
                                       (256, 512, 1024, torch.bfloat16)])
def test_mxfp8(qlib, oracle, m, n, k, out):
    a, b, order = mxfp8_case(oracle, m, n, k)
    dev = torch.device("cuda")
    t = lambda arr: torch.from_numpy(arr).to(dev)
    c = torch.full((m, n), float("nan"), dtype=out, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    qlib.gemm_mxfp8_raw(t(a[0]), t(a[1]), t(b[0]), t(b[1]), c, m, n, k, 1, status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, code
    av, asf = oracle.mxfp8_decode(a[0], a[1], m, k, order)
    bv, bsf = oracle.mxfp8_decode(b[0], b[1], n, k, order)
    ref = oracle.gemm(av, bv, asf, bsf, m, n, k, 32)
    check_gemm(c.float().cpu().numpy(), ref, bf16=(out == torch.bfloat16))


@pytest.mark.parametrize("m,out", [(1, torch.float32), (64, torch.float32), (100, torch.bfloat16),
                                   (128, torch.float32)])
def test_mxfp8_small_m(qlib, oracle, m, out):
    """MXFP8 with m <= 128 runs the single-CTA kernel (gemm_blockscaled.cu,
    tcgen05.cp scale copies) by default; ragged n, several K blocks."""
    n, k = 1000, 1024
    a, b, order = mxfp8_case(oracle, m, n, k)
    dev = torch.device("cuda")
    t = lambda arr: torch.from_numpy(arr).to(dev)
    c = torch.full((m, n), float("nan"), dtype=out, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    qlib.gemm_mxfp8_raw(t(a[0]), t(a[1]), t(b[0]), t(b[1]), c, m, n, k, 1, status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, code
    av, asf = oracle.mxfp8_decode(a[0], a[1], m, k, order)
    bv, bsf = oracle.mxfp8_decode(b[0], b[1], n, k, order)
    ref = oracle.gemm(av, bv, asf, bsf, m, n, k, 32)
    check_gemm(c.float().cpu().numpy(), ref, bf16=(out == torch.bfloat16))


def test_end_to_end_device_quantize(qlib, oracle):
    """Quantise on the device, GEMM on the device, compare with the oracle's
    quantise + O2 on the same fp32 inputs."""
    m, n, k = 256, 512, 512
    xa = oracle.normal(m * k, 1).reshape(m, k)
    xb = oracle.normal(n * k, 2).reshape(n, k)
    A = qlib.make_nvfp4(torch.from_numpy(xa).cuda())
    B = qlib.make_nvfp4(torch.from_numpy(xb).cuda())
    c = qlib.block_scaled_gemm(A, B, torch.float32)
    torch.cuda.synchronize()
    a, b = oracle.nvfp4_mma(xa, 0), oracle.nvfp4_mma(xb, 0)
    check_gemm(c.cpu().numpy(), oracle_nvfp4(oracle, a, b, m, n, k, 0))
