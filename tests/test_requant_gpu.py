"""GPU parity: the NVFP4 GEMM with the output requantised to NVFP4 in its
epilogue (qg_gemm_nvfp4_requant, the B200 counterpart of the reference's tc6
fused epilogue, GEMMsm110/include/backends/tc6_nvfp4.cuh:460-503).

Two checks, mirroring the reference's own test of tc6
(GEMMsm110/src/main.cu:150-223):
* bit_exact: the requantised bytes equal O1's block step
  (make_nvfp4_reference, nvfp4_reference.cuh:84-111) applied under the same
  tensor scale to the fp32 output of qg_gemm_nvfp4 on the same operands.
  The fp32 values are the same accumulator, so any byte difference is a
  requantisation error.
* matched: against the oracle GEMM O2, the reconstruction error of the
  device bytes is no worse than that of O1 over the oracle's own output
  (rmse <= 1.1 x ref + 1e-6, max_abs <= 1.25 x ref + 1e-5, main.cu:207-210).
"""
import numpy as np
import pytest
import torch

from test_gemm_gpu import nvfp4_case, oracle_nvfp4

pytestmark = pytest.mark.gpu


def _dev(arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def _operands(qlib, a, b, m, n, k):
    ats = torch.tensor([a[2]], dtype=torch.float32, device="cuda")
    bts = torch.tensor([b[2]], dtype=torch.float32, device="cuda")
    A = qlib.Nvfp4Result(_dev(a[0]), _dev(a[1]), ats, m, k, qlib.LAYOUT_MMA)
    B = qlib.Nvfp4Result(_dev(b[0]), _dev(b[1]), bts, n, k, qlib.LAYOUT_MMA)
    return A, B


def _reconstruct(oracle, q, sf, ts, n_elems):
    dec_e2m1 = np.array([oracle.L.qgo_decode_e2m1(i) for i in range(16)], np.float32)
    dec_e4m3 = np.array([oracle.L.qgo_decode_e4m3_positive(i) for i in range(256)], np.float32)
    nib = np.empty(q.size * 2, np.uint8)
    nib[0::2] = q >> 4
    nib[1::2] = q & 15
    nib = nib[:n_elems]
    scale = np.repeat(dec_e4m3[sf], 16)[:n_elems]
    return dec_e2m1[nib] * scale * np.float32(ts)


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (512, 768, 512), (130, 272, 128),
                                   (192, 80, 96)])
def test_requant_bit_exact(qlib, oracle, m, n, k):
    a, b, order = nvfp4_case(oracle, qlib, m, n, k)
    A, B = _operands(qlib, a, b, m, n, k)
    c32 = qlib.block_scaled_gemm(A, B, torch.float32)
    c = c32.cpu().numpy()
    amax = float(np.max(np.abs(c)))
    ts = np.float32(amax) / np.float32(2688.0)
    out_ts = torch.tensor([ts], dtype=torch.float32, device="cuda")
    ref_q, ref_sf = oracle.nvfp4_with_ts(c, ts)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for layout in (qlib.LAYOUT_REF_LINEAR, qlib.LAYOUT_MMA, qlib.LAYOUT_MMA_KMAJOR):
        out_amax = torch.zeros(1, dtype=torch.int32, device="cuda")
        r = qlib.gemm_nvfp4_requant(A, B, out_ts, layout, out_amax=out_amax, status=status)
        rc, code = qlib.read_status(status)
        assert rc == qlib.OK, f"device status {code}"
        got_q = r.quantized.cpu().numpy()
        got_sf = r.block_scales.cpu().numpy()
        if layout == qlib.LAYOUT_REF_LINEAR:
            want_q, want_sf = ref_q, ref_sf
        else:
            want_q, want_sf = oracle.linear_to_mma(ref_q, ref_sf, m, n,
                                                   0 if layout == qlib.LAYOUT_MMA else 1)
        assert np.array_equal(got_q, want_q), f"layout {layout}: value bytes differ"
        assert np.array_equal(got_sf, want_sf), f"layout {layout}: scale bytes differ"
        got_amax = np.array([out_amax.item()], np.int32).view(np.float32)[0]
        assert got_amax == np.float32(amax)


def test_requant_matches_oracle_gemm(qlib, oracle):
    m = n = k = 256
    a, b, order = nvfp4_case(oracle, qlib, m, n, k)
    A, B = _operands(qlib, a, b, m, n, k)
    ref = oracle_nvfp4(oracle, a, b, m, n, k, order).astype(np.float32)
    rq, rsf, rts = oracle.nvfp4_reference(ref)
    out_ts = torch.tensor([rts], dtype=torch.float32, device="cuda")
    r = qlib.gemm_nvfp4_requant(A, B, out_ts, qlib.LAYOUT_REF_LINEAR)
    got = _reconstruct(oracle, r.quantized.cpu().numpy(), r.block_scales.cpu().numpy(), rts,
                       m * n)
    want = _reconstruct(oracle, rq, rsf, rts, m * n)
    flat = ref.ravel()
    rmse_got = float(np.sqrt(np.mean((got.astype(np.float64) - flat) ** 2)))
    rmse_ref = float(np.sqrt(np.mean((want.astype(np.float64) - flat) ** 2)))
    max_got = float(np.max(np.abs(got - flat)))
    max_ref = float(np.max(np.abs(want - flat)))
    assert rmse_got <= rmse_ref * 1.10 + 1e-6, (rmse_got, rmse_ref)
    assert max_got <= max_ref * 1.25 + 1e-5, (max_got, max_ref)


def test_requant_output_feeds_next_gemm(qlib, oracle):
    """The MMA-layout output is a valid A operand (K = n) for the next GEMM:
    equal to the GEMM over the oracle's quantisation of the fp32 output."""
    m, n, k, n2 = 256, 512, 256, 256
    a, b, order = nvfp4_case(oracle, qlib, m, n, k)
    A, B = _operands(qlib, a, b, m, n, k)
    c = qlib.block_scaled_gemm(A, B, torch.float32).cpu().numpy()
    ts = np.float32(np.max(np.abs(c))) / np.float32(2688.0)
    out_ts = torch.tensor([ts], dtype=torch.float32, device="cuda")
    A2 = qlib.gemm_nvfp4_requant(A, B, out_ts, qlib.LAYOUT_MMA)
    xw = oracle.normal(n2 * n, 77).reshape(n2, n)
    qw, sw, tw = oracle.nvfp4_mma(xw, 0)
    W = qlib.Nvfp4Result(_dev(qw), _dev(sw), torch.tensor([tw], dtype=torch.float32,
                                                            device="cuda"), n2, n, qlib.LAYOUT_MMA)
    got = qlib.block_scaled_gemm(A2, W, torch.float32).cpu().numpy()
    q1, s1 = oracle.nvfp4_with_ts(c, ts)
    qa, sa = oracle.linear_to_mma(q1, s1, m, n, 0)
    want = oracle_nvfp4(oracle, (qa, sa, ts), (qw, sw, tw), m, n2, n, 0)
    from helpers import check_gemm
    check_gemm(got, want)


def test_requant_rejects_bad_args(qlib):
    m = n = k = 128
    A = qlib.Nvfp4Result(torch.zeros(m * k // 2, dtype=torch.uint8, device="cuda"),
                         torch.zeros(qlib.sm1xx_scale_storage_size(m, k, 16), dtype=torch.uint8,
                                     device="cuda"), None, m, k, qlib.LAYOUT_MMA)
    q = torch.zeros(m * n // 2, dtype=torch.uint8, device="cuda")
    sf = torch.zeros(m * n // 16, dtype=torch.uint8, device="cuda")
    L = qlib.lib()
    p = A.quantized.data_ptr()
    s = A.block_scales.data_ptr()
    assert L.qg_gemm_nvfp4_requant(p, s, None, p, s, None, None, q.data_ptr(), sf.data_ptr(), 0,
                                   None, m, 24, k, 1, None, None) == qlib.ERR_SHAPE
    assert L.qg_gemm_nvfp4_requant(p, s, None, p, s, None, None, q.data_ptr(), sf.data_ptr(), 7,
                                   None, m, n, k, 1, None, None) == qlib.ERR_LAYOUT
    assert L.qg_gemm_nvfp4_requant(p, s, None, p, s, None, None, None, sf.data_ptr(), 0,
                                   None, m, n, k, 1, None, None) == qlib.ERR_ARG
    assert L.qg_gemm_nvfp4_requant(p, s, None, p, s, None, None, q.data_ptr() + 8, sf.data_ptr(),
                                   0, None, m, n, k, 1, None, None) == qlib.ERR_ALIGN


def test_e2m1_cvt_exhaustive(qlib):
    """The epilogue's hardware e2m1 conversion equals the restated reference
    encoder (encode_e2m1_rn, GEMMsm110/include/requant/e2m1_encode.cuh:18-44)
    on every non-NaN fp32 bit pattern (NaN is mapped to +0 before it)."""
    out = torch.zeros(3, dtype=torch.int64, device="cuda")
    rc = qlib.lib().qg_selftest_e2m1_cvt(out.data_ptr(), None)
    assert rc == qlib.OK
    bad, bad_nan, last = out.cpu().tolist()
    assert bad == 0, f"{bad} non-NaN mismatches, e.g. bits {last - 1:#010x}"
