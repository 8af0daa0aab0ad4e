"""GPU parity at the benchmarked configurations.

Each case runs the public call at the full benchmarked shape and checks it
against the CPU oracle on a deterministic sample: whole output rows
``s*131 % M`` (the reference's sampling pattern, GEMMsm110/include/
gemm_benchmark.cuh:51-53, widened to whole rows so the per-element bound
1e-3*||oracle row||_2 is the north-star one; the decode GEMM samples output
columns instead, every row being checked).  On the way the quantised operands
are checked too: the tensor scale against amax/(448*6)
(GEMMsm110/include/requant/nvfp4_reference.cuh:66-74) and the bytes of every
sampled row against O1's block rule under that scale
(nvfp4_reference.cuh:84-111), or against the OCP MX rule for MXFP8.  Inputs
are seeded torch.randn on the device (the quantisers read them there; the
oracle reads the host copy of the same fp32 values).
"""
import os

import numpy as np
import pytest
import torch

from helpers import check_gemm

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8


def sample_rows(m: int, count: int) -> list:
    """Whole rows s*131 % m for s < count, plus the last row."""
    return sorted({(s * 131) % m for s in range(count)} | {m - 1})


def dev_normal(rows, k, seed, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, k, generator=g, device="cuda", dtype=torch.float32)
    return x * std if std != 1.0 else x


def nvfp4_checked(oracle, qlib, x, rows_idx, layout):
    """Quantise x (CUDA fp32) on the GPU; check its tensor scale and the
    bytes of rows_idx against O1; return the result and the oracle's logical
    view (values, scales) of those rows."""
    order = 0 if layout == qlib.LAYOUT_MMA else 1
    rows, k = x.shape
    res = qlib.make_nvfp4(x, layout)
    return res, *nvfp4_rows_checked(oracle, res, x, rows_idx, order)


def nvfp4_rows_checked(oracle, res, x, rows_idx, order, amax=None):
    """x: the fp32 rows `res` was quantised from; amax: the absolute maximum
    of the whole tensor the tensor scale came from (default: of x)."""
    rows, k = res.rows, res.k
    amax = np.float32(x.abs().max().item() if amax is None else amax)
    ts = np.float32(res.tensor_scale.item())
    assert ts == (amax / np.float32(2688.0) if amax > 0 else np.float32(1.0)), (ts, amax)
    idx = torch.tensor(rows_idx, device=x.device)
    xr = x[idx].cpu().numpy()
    lq, lsf = oracle.nvfp4_with_ts(xr, float(ts))
    qm, _ = oracle.linear_to_mma(lq, lsf, len(rows_idx), k, 0)
    gq = res.quantized.view(rows, k // 2)[idx].cpu().numpy()
    gsf = res.block_scales.cpu().numpy()
    assert np.array_equal(gq, qm.reshape(len(rows_idx), k // 2)), "NVFP4 values differ from O1"
    assert np.array_equal(oracle.scale_rows(gsf, rows_idx, rows, k, 16, order),
                          lsf.reshape(len(rows_idx), k // 16)), "NVFP4 scales differ from O1"
    q_host = np.zeros(rows * k // 2, np.uint8)
    q_host.reshape(rows, k // 2)[rows_idx] = gq
    return oracle.nvfp4_rows(q_host, gsf, rows_idx, rows, k, order)


def o2_nvfp4(oracle, av, asf, bv, bsf, nrows, n, k, ts_a, ts_b):
    d = oracle.gemm(av, bv, asf, bsf, nrows, n, k, 16, threads=THREADS)
    return d * np.float32(np.float32(ts_a) * np.float32(ts_b))


def test_nvfp4_8192_bf16_sampled_rows(qlib, oracle):
    """NVFP4 8192^3, bf16 output, N(0,1) operands."""
    m = n = k = 8192
    rows = sample_rows(m, 64)
    xa, xb = dev_normal(m, k, 20260817), dev_normal(n, k, 20260817 ^ 0xBB67AE85)
    A, av, asf = nvfp4_checked(oracle, qlib, xa, rows, qlib.LAYOUT_MMA)
    B, bv, bsf = nvfp4_checked(oracle, qlib, xb, list(range(n)), qlib.LAYOUT_MMA)
    del xa, xb
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    c = qlib.block_scaled_gemm(A, B, torch.bfloat16, status=status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, f"device status {code}"
    got = c[torch.tensor(rows, device="cuda")].float().cpu().numpy()
    ref = o2_nvfp4(oracle, av, asf, bv, bsf, len(rows), n, k, A.tensor_scale.item(),
                   B.tensor_scale.item())
    check_gemm(got, ref, bf16=True)


def test_mxfp8_ffn_bf16_sampled_rows(qlib, oracle):
    """MXFP8 4096 x 14336 x 4096, A N(0,1), B N(0,0.02),
    bf16 output."""
    m, n, k = 4096, 14336, 4096
    rows = sample_rows(m, 48)
    xa, xb = dev_normal(m, k, 31), dev_normal(n, k, 32, 0.02)
    A, B = qlib.make_mxfp8(xa), qlib.make_mxfp8(xb)
    idx = torch.tensor(rows, device="cuda")
    # Quantiser bytes: the sampled rows of A and all of B against the
    # oracle's OCP MX rule (linear scales, order -1).
    qa_ref, sa_ref = oracle.mxfp8(xa[idx].cpu().numpy(), -1)
    qb_ref, sb_ref = oracle.mxfp8(xb.cpu().numpy(), -1)
    del xa, xb
    ga = A.quantized.view(m, k)[idx].cpu().numpy()
    gasf, gb, gbsf = A.block_scales.cpu().numpy(), B.quantized.cpu().numpy(), B.block_scales.cpu().numpy()
    assert np.array_equal(ga.ravel(), qa_ref)
    assert np.array_equal(oracle.scale_rows(gasf, rows, m, k, 32, 0).ravel(), sa_ref)
    assert np.array_equal(gb, qb_ref)
    assert np.array_equal(oracle.scale_rows(gbsf, range(n), n, k, 32, 0).ravel(), sb_ref)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    c = qlib.block_scaled_gemm(A, B, torch.bfloat16, status=status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, f"device status {code}"
    qa_full = np.zeros(m * k, np.uint8)
    qa_full.reshape(m, k)[rows] = ga
    av, asf = oracle.mxfp8_rows(qa_full, gasf, rows, m, k, 0)
    bv, bsf = oracle.mxfp8_decode(gb, gbsf, n, k, 0)
    ref = oracle.gemm(av, bv, asf, bsf, len(rows), n, k, 32, threads=THREADS)
    check_gemm(c[idx].float().cpu().numpy(), ref, bf16=True)


def test_colpar_shards_16384x53248x8192(qlib, oracle):
    """BASELINE config 5 on one GPU: B (53248 x 8192) quantised once, two of
    its 8-way column shards (first and last) cut with colpar.shard_rows and
    multiplied by the broadcast A; sampled rows of each shard's output
    against O2."""
    from cuda_optimazation_b200 import colpar
    m, n, k, world = 16384, 53248, 8192, 8
    rows = sample_rows(m, 32)
    xa = dev_normal(m, k, 41)
    A, av, asf = nvfp4_checked(oracle, qlib, xa, rows, qlib.LAYOUT_MMA_KMAJOR)
    del xa
    xb = dev_normal(n, k, 42)
    B = qlib.make_nvfp4(xb, qlib.LAYOUT_MMA_KMAJOR)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for rank in (0, world - 1):
        lo, hi = colpar.shard_range(n, world, rank)
        Bs = colpar.shard_rows(B, lo, hi)
        assert (Bs.rows, lo % 256) == (hi - lo, 0)
        # The shard's bytes are O1 of its rows under the FULL B tensor scale.
        bv, bsf = nvfp4_rows_checked(oracle, Bs, xb[lo:hi], list(range(hi - lo)), 1,
                                     amax=xb.abs().max().item())
        c = qlib.block_scaled_gemm(A, Bs, torch.bfloat16, status=status)
        rc, code = qlib.read_status(status)
        assert rc == qlib.OK, f"device status {code}"
        got = c[torch.tensor(rows, device="cuda")].float().cpu().numpy()
        ref = o2_nvfp4(oracle, av, asf, bv, bsf, len(rows), hi - lo, k, A.tensor_scale.item(),
                       Bs.tensor_scale.item())
        check_gemm(got, ref, bf16=True)


@pytest.fixture(scope="module")
def decode_weights(qlib):
    """BASELINE config 4 weights: N(0, 0.02), 28672 x 8192, pre-quantised."""
    n, k = 28672, 8192
    xw = dev_normal(n, k, 7, 0.02)
    W = qlib.make_nvfp4(xw)
    return xw, W


@pytest.mark.parametrize("m", [64, 128])
def test_decode_config_full_n_sampled_columns(qlib, oracle, decode_weights, m):
    """BASELINE config 4 at m = 64 and 128 (m = 16 is in test_skinny_gpu):
    bf16 activations N(0,1) with every 1000th element x50, activation
    quantisation fused in the call; every output row, columns sampled in
    every weight tile."""
    xw, W = decode_weights
    n, k = W.rows, W.k
    cols = sorted(set(range(0, n, 53)) | set(range(n - 128, n)))
    x = oracle.normal(m * k, 900 + m).reshape(m, k)
    x.reshape(-1)[::1000] *= 50.0
    xb = torch.from_numpy(x).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    c = qlib.gemm_nvfp4_skinny(xb.cuda(), W, torch.bfloat16, status=status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, f"device status {code}"
    qa, sa, ta = oracle.nvfp4_mma(xb.float().numpy(), 0)
    av, asf = oracle.nvfp4_decode(qa, sa, m, k)
    wv, wsf = nvfp4_rows_checked(oracle, W, xw, cols, 0)
    ref = o2_nvfp4(oracle, av, asf, wv, wsf, m, len(cols), k, ta, W.tensor_scale.item())
    got = c[:, torch.tensor(cols, device="cuda")].float().cpu().numpy()
    check_gemm(got, ref, bf16=True)
