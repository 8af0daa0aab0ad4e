"""GPU parity for MXFP4 (e2m1 values, ue8m0 scale per 32 K elements; the
reference's MXFP4 rows run CUTLASS example 72a,
GEMMquant_sm110/scripts/run_quant_gemm_1024.py:54-73): the quantizer bit for
bit against the oracle's OCP MX restatement (parity unpinned: the reference
has no MXFP4 quantizer), and the tcgen05 GEMM (kind::mxf4nvf4.block32)
against O2 (block_scaled_reference_mnk, SV = 32) within the stated
tolerance (tests/helpers.py)."""
import numpy as np
import pytest
import torch

from helpers import check_gemm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout,order", [(0, -1), (1, 0), (2, 1)])
@pytest.mark.parametrize("shape", [(128, 256), (130, 96), (1, 32), (300, 1024)])
def test_mxfp4_quantize_bit_exact(qlib, oracle, layout, order, shape):
    rows, k = shape
    x = oracle.normal(rows * k, 23).reshape(rows, k)
    if rows > 1:
        x[0, :32] *= 1e-30  # tiny block: exponent clamps toward -127
        x[1, :32] = 0.0     # all-zero block -> code 0
        if k >= 64:  # a block spanning 2^31 of dynamic range
            x[1, 32:64] = 6.0 * 2.0 ** np.arange(32)
    x.ravel()[::97] *= 40.0  # outliers
    for dt in (torch.float32, torch.bfloat16):
        xt = torch.from_numpy(x).cuda().to(dt).contiguous()
        q, sf = oracle.mxfp4(xt.float().cpu().numpy(), order)
        r = qlib.make_mxfp4(xt, layout)
        torch.cuda.synchronize()
        assert np.array_equal(r.quantized.cpu().numpy(), q), f"{dt} values"
        assert np.array_equal(r.block_scales.cpu().numpy(), sf), f"{dt} scales"


def mxfp4_case(oracle, m, n, k, layout=1):
    order = 0 if layout == 1 else 1
    xa = oracle.normal(m * k, 31).reshape(m, k)
    xb = oracle.normal(n * k, 32, 0.0, 0.02).reshape(n, k)
    return oracle.mxfp4(xa, order), oracle.mxfp4(xb, order), order


@pytest.mark.parametrize("m,n,k,out,layout", [(256, 256, 256, torch.float32, 1),
                                              (130, 300, 544, torch.float32, 1),
                                              (64, 256, 96, torch.float32, 1),
                                              (512, 512, 1024, torch.float32, 2),
                                              (256, 512, 1024, torch.bfloat16, 1)])
def test_mxfp4_gemm(qlib, oracle, m, n, k, out, layout):
    a, b, order = mxfp4_case(oracle, m, n, k, layout)
    dev = torch.device("cuda")
    t = lambda arr: torch.from_numpy(arr).to(dev)
    c = torch.full((m, n), float("nan"), dtype=out, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    qlib.gemm_mxfp4_raw(t(a[0]), t(a[1]), t(b[0]), t(b[1]), c, m, n, k, layout, status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, code
    av, asf = oracle.mxfp4_decode(a[0], a[1], m, k, order)
    bv, bsf = oracle.mxfp4_decode(b[0], b[1], n, k, order)
    ref = oracle.gemm(av, bv, asf, bsf, m, n, k, 32)
    check_gemm(c.float().cpu().numpy(), ref, bf16=(out == torch.bfloat16))


def test_mxfp4_device_quantize_then_gemm(qlib, oracle):
    m, n, k = 256, 512, 512
    xa = oracle.normal(m * k, 5).reshape(m, k)
    xb = oracle.normal(n * k, 6).reshape(n, k)
    A = qlib.make_mxfp4(torch.from_numpy(xa).cuda())
    B = qlib.make_mxfp4(torch.from_numpy(xb).cuda())
    c = qlib.block_scaled_gemm(A, B, torch.float32).cpu().numpy()
    (qa, sa), (qb, sb) = oracle.mxfp4(xa, 0), oracle.mxfp4(xb, 0)
    av, asf = oracle.mxfp4_decode(qa, sa, m, k, 0)
    bv, bsf = oracle.mxfp4_decode(qb, sb, n, k, 0)
    check_gemm(c, oracle.gemm(av, bv, asf, bsf, m, n, k, 32))
