"""GPU parity: decode-shaped NVFP4 GEMM with fused activation quantisation
(qg_gemm_nvfp4_skinny) vs the oracle's quantiser + O2."""
import numpy as np
import pytest
import torch

from helpers import check_gemm

pytestmark = pytest.mark.gpu


def activations(oracle, m, k, seed):
    """N(0,1) with 0.1% outliers x50 (every 1000th element), bf16-rounded."""
    x = oracle.normal(m * k, seed).reshape(m, k)
    x.reshape(-1)[::1000] *= 50.0
    return torch.from_numpy(x).to(torch.bfloat16)


def run_case(qlib, oracle, m, n, k, out_dtype=torch.float32, cols=None):
    xb = activations(oracle, m, k, 100 + m)
    xw = oracle.normal(n * k, 7, 0.0, 0.02).reshape(n, k)
    W = qlib.make_nvfp4(torch.from_numpy(xw).cuda())
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    c = qlib.gemm_nvfp4_skinny(xb.cuda(), W, out_dtype, status=status)
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, code
    got = c.float().cpu().numpy()
    # Oracle: quantise the (bf16-exact) activations and the weights, O2.
    xa = xb.float().numpy()
    qa, sa, ta = oracle.nvfp4_mma(xa, 0)
    qw, sw, tw = oracle.nvfp4_mma(xw, 0)
    av, asf = oracle.nvfp4_decode(qa, sa, m, k)
    wv, wsf = oracle.nvfp4_decode(qw, sw, n, k)
    if cols is not None:
        wv = wv.reshape(n, k)[cols].ravel()
        wsf = wsf.reshape(n, k // 16)[cols].ravel()
        got = got[:, cols]
    nn = n if cols is None else len(cols)
    ref = oracle.gemm(av, np.ascontiguousarray(wv), asf, np.ascontiguousarray(wsf), m, nn, k, 16)
    ref = ref * np.float32(np.float32(ta) * np.float32(tw))
    return check_gemm(got, ref, bf16=(out_dtype == torch.bfloat16))


@pytest.mark.parametrize("m", [1, 16, 37, 64, 128])
def test_skinny_fp32(qlib, oracle, m):
    run_case(qlib, oracle, m, 1000, 1024)


@pytest.mark.parametrize("m,n,k", [(16, 4096, 544), (64, 384, 8192), (128, 2048, 256)])
def test_skinny_shapes_bf16(qlib, oracle, m, n, k):
    run_case(qlib, oracle, m, n, k, torch.bfloat16)


def test_skinny_decode_config_sampled_columns(qlib, oracle):
    """BASELINE config 4 shape (M=16, N=28672, K=8192) with the oracle on a
    deterministic subset of output columns spread over every weight tile."""
    cols = np.unique(np.concatenate([np.arange(0, 28672, 97), np.arange(28544, 28672)]))
    run_case(qlib, oracle, 16, 28672, 8192, torch.float32, cols=cols)


def test_skinny_rejects_large_m(qlib):
    L = qlib.lib()
    d = torch.empty(16, dtype=torch.uint8, device="cuda")
    rc = L.qg_gemm_nvfp4_skinny(d.data_ptr(), 1, 129, d.data_ptr(), d.data_ptr(), None,
                                d.data_ptr(), 1, 256, 256, 256, 1, d.data_ptr(), 1 << 30, None,
                                None)
    assert rc == qlib.ERR_SHAPE


def test_skinny_fp32_activations(qlib, oracle):
    """fp32 x (the other input dtype of the in-kernel quantiser)."""
    m, n, k = 24, 640, 2048
    xa = oracle.normal(m * k, 321).reshape(m, k)
    xw = oracle.normal(n * k, 8, 0.0, 0.02).reshape(n, k)
    W = qlib.make_nvfp4(torch.from_numpy(xw).cuda())
    got = qlib.gemm_nvfp4_skinny(torch.from_numpy(xa).cuda(), W, torch.float32).cpu().numpy()
    qa, sa, ta = oracle.nvfp4_mma(xa, 0)
    qw, sw, tw = oracle.nvfp4_mma(xw, 0)
    av, asf = oracle.nvfp4_decode(qa, sa, m, k)
    wv, wsf = oracle.nvfp4_decode(qw, sw, n, k)
    ref = oracle.gemm(av, wv, asf, wsf, m, n, k, 16) * np.float32(np.float32(ta) * np.float32(tw))
    check_gemm(got, ref)


def test_skinny_workspace_reuse_and_determinism(qlib, oracle):
    """One workspace across calls with different activations: the tile
    counters are re-zeroed by every call's quantiser, and split tiles are
    summed in a fixed order, so a repeated call is bit-identical."""
    m, n, k = 16, 28672, 2048
    xw = oracle.normal(n * k, 9, 0.0, 0.02).reshape(n, k)
    W = qlib.make_nvfp4(torch.from_numpy(xw).cuda())
    ws = qlib.skinny_workspace(m, n, k, "cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    xs = [activations(oracle, m, k, s).cuda() for s in (1, 2)]
    outs = [qlib.gemm_nvfp4_skinny(xs[i % 2], W, torch.float32, workspace=ws, status=status)
            for i in range(4)]
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, code
    assert torch.equal(outs[0], outs[2]) and torch.equal(outs[1], outs[3])
    assert not torch.equal(outs[0], outs[1])
    # A fresh workspace gives the same bits.
    fresh = qlib.gemm_nvfp4_skinny(xs[0], W, torch.float32)
    assert torch.equal(fresh, outs[0])


def test_skinny_workspace_shared_across_shapes(qlib, oracle):
    """One workspace sized for the largest call serves smaller m and k: the
    activation scales left by a larger call (rows >= m, columns >= k/16) are
    never rewritten and must not change the smaller call's result."""
    n = 4096
    ws = qlib.skinny_workspace(128, n, 2048, "cuda")
    out = {}
    for m, k in ((128, 2048), (16, 1056), (64, 2048), (16, 1056)):
        xw = oracle.normal(n * k, 11, 0.0, 0.02).reshape(n, k)
        W = qlib.make_nvfp4(torch.from_numpy(xw).cuda())
        x = activations(oracle, m, k, 3).cuda()
        got = qlib.gemm_nvfp4_skinny(x, W, torch.float32, workspace=ws)
        fresh = qlib.gemm_nvfp4_skinny(x, W, torch.float32)
        assert torch.equal(got, fresh), (m, k)
        out.setdefault((m, k), []).append(got)
    assert torch.equal(*out[(16, 1056)])


@pytest.mark.parametrize("m,n,k", [(16, 19968, 1024),   # 156 tiles: too few split units, all stream-K
                                   (32, 51200, 1024),   # 400 tiles: 2 whole tiles per CTA + split rest
                                   (64, 38016, 512)])   # 297 tiles, one unit each: all stream-K
def test_skinny_schedules(qlib, oracle, m, n, k):
    """Both work decompositions (whole tiles + stream-K remainder, and pure
    stream-K when the remainder has fewer units than CTAs), sampled columns
    in every weight tile."""
    cols = np.unique(np.concatenate([np.arange(0, n, 61), np.arange(n - 128, n)]))
    run_case(qlib, oracle, m, n, k, torch.bfloat16, cols=cols)


@pytest.mark.parametrize("m,n,out", [(128, 28736, torch.bfloat16), (100, 28800, torch.float32),
                                     (64, 28736, torch.float32), (40, 28800, torch.bfloat16)])
def test_skinny_wide_whole_tiles_ragged_n(qlib, oracle, m, n, out):
    """m > 32 at a decode-sized N takes whole 512-row tiles on CTA pairs
    (two 128-row halves per CTA); N = 28736 and 28800 (57 pair tiles) leave
    the last tile's first CTA partly past the weights' end and its second
    CTA wholly past it."""
    cols = np.unique(np.concatenate([np.arange(0, n, 89), np.arange(n - 300, n)]))
    run_case(qlib, oracle, m, n, 1024, out, cols=cols)


def test_skinny_chained_calls_read_previous_output(qlib, oracle):
    """A decode call whose activations are the previous call's output on the
    same stream (its amax kernel must start only after that GEMM has
    finished; the quantiser and GEMM launch early and wait on it): the
    chained result equals the same call made after a device synchronise."""
    m, k, n1, n2 = 16, 1024, 4096, 2048
    W1 = qlib.make_nvfp4(torch.from_numpy(oracle.normal(n1 * k, 21, 0.0, 0.02).reshape(n1, k)).cuda())
    W2 = qlib.make_nvfp4(torch.from_numpy(oracle.normal(n2 * n1, 22, 0.0, 0.02).reshape(n2, n1)).cuda())
    x = activations(oracle, m, k, 5).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws1 = qlib.skinny_workspace(m, n1, k, "cuda")
    ws2 = qlib.skinny_workspace(m, n2, n1, "cuda")
    chained = []
    for _ in range(3):
        y1 = qlib.gemm_nvfp4_skinny(x * 2.0, W1, torch.bfloat16, workspace=ws1, status=status)
        chained.append(qlib.gemm_nvfp4_skinny(y1, W2, torch.float32, workspace=ws2, status=status))
    torch.cuda.synchronize()
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK, code
    y1 = qlib.gemm_nvfp4_skinny(x * 2.0, W1, torch.bfloat16, workspace=ws1, status=status)
    torch.cuda.synchronize()
    ref = qlib.gemm_nvfp4_skinny(y1.clone(), W2, torch.float32, workspace=ws2, status=status)
    torch.cuda.synchronize()
    for c in chained:
        assert torch.equal(c, ref)


@pytest.mark.parametrize("m,k,out", [(64, 1056, torch.bfloat16), (128, 2080, torch.float32),
                                     (33, 8192, torch.bfloat16)])
def test_skinny_pair_tiles(qlib, oracle, m, k, out):
    """m in (32, 128] at a decode-sized N runs on CTA pairs (one 512-row
    weight tile per pair, each CTA loading half of the activation rows):
    K not a multiple of the 256-element stage (the last stage partly past
    the operands' end), fp32 and bf16 output, and the fewest rows that take
    the pairs; sampled columns in every tile, and repeated calls give the
    same bits."""
    n = 28672
    cols = np.unique(np.concatenate([np.arange(0, n, 127), np.arange(n - 512, n)]))
    run_case(qlib, oracle, m, n, k, out, cols=cols)
    xw = oracle.normal(n * k, 7, 0.0, 0.02).reshape(n, k)
    W = qlib.make_nvfp4(torch.from_numpy(xw).cuda())
    x = activations(oracle, m, k, 100 + m).cuda()
    a = qlib.gemm_nvfp4_skinny(x, W, out)
    b = qlib.gemm_nvfp4_skinny(x, W, out)
    assert torch.equal(a, b)
