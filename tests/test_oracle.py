"""CPU tests: the oracle against the reference's known-answer tests and the
reference's own host code (oracle/_ref), plus the committed golden vectors."""
import math
from pathlib import Path

import numpy as np
import pytest

import oracle as om

GOLDEN = Path(__file__).resolve().parent / "golden"


# GEMMsm110/tests/requant_epilogue_benchmark.cu:54-73
E2M1_KATS = [(0.0, 0x0), (-0.0, 0x8), (0.25, 0x0), (-0.25, 0x8), (0.75, 0x2), (-0.75, 0xa),
             (1.25, 0x2), (-1.25, 0xa), (1.75, 0x4), (-1.75, 0xc), (2.5, 0x4), (-2.5, 0xc),
             (3.5, 0x6), (-3.5, 0xe), (5.0, 0x6), (-5.0, 0xe),
             (math.inf, 0x7), (-math.inf, 0xf), (math.nan, 0x0)]


@pytest.mark.parametrize("v,code", E2M1_KATS)
def test_e2m1_kat(oracle, v, code):
    assert oracle.L.qgo_encode_e2m1(v) == code


def test_pack_kat(oracle):
    # requant_epilogue_benchmark.cu:73: pack_e2m1x2(0x2, 0xb) == 0x2b
    assert oracle.L.qgo_pack_e2m1x2(0x2, 0xB) == 0x2B


def test_scale_layout_kats(oracle):
    # cutlass-gemm-cpp-guide/tests/host/test_references.cpp:28-43
    L = oracle.L
    assert L.qgo_scale_storage_size(128, 128, 32) == 512
    assert L.qgo_scale_offset(0, 0, 128, 128, 32, 0) == 0
    assert L.qgo_scale_offset(0, 32, 128, 128, 32, 0) == 1
    assert L.qgo_scale_offset(32, 0, 128, 128, 32, 0) == 4
    assert L.qgo_scale_offset(1, 0, 128, 128, 32, 0) == 16
    assert L.qgo_scale_offset(127, 127, 128, 128, 32, 0) == 511
    assert L.qgo_scale_storage_size(129, 129, 32) == 2048


def test_scale_layout_orders_agree_on_single_block(oracle):
    L = oracle.L
    for mn in range(0, 128, 7):
        for kk in range(0, 4096, 16 * 5):
            assert L.qgo_scale_offset(mn, kk, 128, 4096, 16, 0) == L.qgo_scale_offset(
                mn, kk, 128, 4096, 16, 1)
    for mn in range(0, 1024, 13):
        for kk in range(0, 64, 16):
            assert L.qgo_scale_offset(mn, kk, 1024, 64, 16, 0) == L.qgo_scale_offset(
                mn, kk, 1024, 64, 16, 1)


def test_block_scaled_kat(oracle):
    # test_references.cpp:45-53: 1x1x4, SV 2 -> 931
    a = np.array([1, 2, 3, 4], np.float32)
    b = np.array([5, 6, 7, 8], np.float32)
    sfa = np.array([2, 3], np.float32)
    sfb = np.array([4, 5], np.float32)
    d = oracle.gemm(a, b, sfa, sfb, 1, 1, 4, 2, threads=1)
    assert d[0, 0] == 931.0


def test_dense_kat(oracle):
    # test_references.cpp:19-26 (dense oracle == block-scaled with unit scales)
    a = np.array([1, 2, 3, 4, 5, 6], np.float32)
    b = np.array([7, 8, 9, 1, 2, 3], np.float32)
    ones = np.ones(2 * 3, np.float32)
    d = oracle.gemm(a, b, ones, ones, 2, 2, 3, 1, threads=1)
    assert d.ravel().tolist() == [50.0, 14.0, 122.0, 32.0]


def test_e4m3_round_up_matches_scan(oracle):
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.uniform(0, 500, 20000), np.exp(rng.uniform(-25, 7, 20000)),
        [0.0, -1.0, 448.0, 448.0001, 1e-30, 2.0 ** -9, 2.0 ** -6, 2.0 ** -10, 1e38],
    ]).astype(np.float32)
    for v in vals:
        c = oracle.L.qgo_encode_e4m3_round_up(float(v))
        if v > 0 and v <= 448:
            assert oracle.L.qgo_decode_e4m3_positive(c) >= v
            if c > 1:
                assert oracle.L.qgo_decode_e4m3_positive(c - 1) < v


needs_ref = pytest.mark.skipif(not om.reference_available(),
                               reason="reference checkout not present")


@needs_ref
@pytest.mark.parametrize("dist", om.DISTRIBUTIONS)
@pytest.mark.parametrize("shape", [(256, 256), (1024, 1024)])
def test_nvfp4_oracle_matches_reference(oracle, dist, shape):
    ref = om.Reference()
    x = oracle.requant_dist(shape[0] * shape[1], dist, 1234)
    q0, s0, t0 = oracle.nvfp4_reference(x)
    q1, s1, t1 = ref.nvfp4_reference(x)
    assert t0 == t1
    assert np.array_equal(q0, q1)
    assert np.array_equal(s0, s1)


@needs_ref
def test_nvfp4_oracle_ragged_matches_reference(oracle):
    ref = om.Reference()
    for n in (1, 15, 17, 1000, 4099):
        x = oracle.requant_dist(n, "normal", 7 + n)
        a, b = oracle.nvfp4_reference(x), ref.nvfp4_reference(x)
        assert a[2] == b[2] and np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@needs_ref
def test_codecs_match_reference(oracle):
    ref = om.Reference()
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.normal(0, 4, 50000), rng.uniform(-7, 7, 50000),
                           np.arange(-6.5, 6.5, 0.125)]).astype(np.float32)
    for v in vals:
        assert oracle.L.qgo_encode_e2m1(float(v)) == ref.L.qgr_encode_e2m1(float(v))
    for v in np.exp(rng.uniform(-25, 7, 20000)).astype(np.float32):
        assert oracle.L.qgo_encode_e4m3_round_up(float(v)) == ref.L.qgr_encode_e4m3_round_up(float(v))


@needs_ref
def test_scale_offset_matches_reference(oracle):
    ref = om.Reference()
    for (mn_ext, k_ext, sv) in [(128, 128, 32), (129, 129, 32), (384, 1024, 16), (1000, 4096, 16)]:
        assert oracle.L.qgo_scale_storage_size(mn_ext, k_ext, sv) == ref.L.qgr_scale_storage_size(
            mn_ext, k_ext, sv)
        for mn in range(0, mn_ext, 37):
            for kk in range(0, k_ext, sv * 3):
                assert oracle.L.qgo_scale_offset(mn, kk, mn_ext, k_ext, sv, 0) == \
                    ref.L.qgr_scale_offset(mn, kk, mn_ext, k_ext, sv)


@needs_ref
def test_block_scaled_gemm_matches_reference(oracle):
    ref = om.Reference()
    m, n, k = 40, 24, 256
    x = oracle.normal(m * k, 3)
    w = oracle.normal(n * k, 4)
    qa, sa, _ = oracle.nvfp4_mma(x.reshape(m, k))
    qb, sb, _ = oracle.nvfp4_mma(w.reshape(n, k))
    av, asf = oracle.nvfp4_decode(qa, sa, m, k)
    bv, bsf = oracle.nvfp4_decode(qb, sb, n, k)
    d0 = oracle.gemm(av, bv, asf, bsf, m, n, k, 16)
    d1 = ref.gemm(av, bv, asf, bsf, m, n, k, 16)
    assert np.array_equal(d0, d1)


def test_golden_vectors(oracle):
    """The committed fixtures were produced by the reference's own code
    (tests/golden/make_golden.py); the oracle must reproduce them."""
    z = np.load(GOLDEN / "nvfp4_requant_64x64.npz")
    for dist in om.DISTRIBUTIONS:
        x = z[f"{dist}_x"]
        q, sf, ts = oracle.nvfp4_reference(x)
        assert np.array_equal(q, z[f"{dist}_q"]), dist
        assert np.array_equal(sf, z[f"{dist}_sf"]), dist
        assert np.float32(ts) == z[f"{dist}_ts"][0], dist
    g = np.load(GOLDEN / "block_scaled_gemm_48x40x256.npz")
    d = oracle.gemm(g["a"], g["b"], g["sfa"], g["sfb"], 48, 40, 256, 16)
    assert np.array_equal(d, g["d"])


def test_mxfp8_oracle_properties(oracle):
    x = oracle.normal(64 * 256, 11).reshape(64, 256)
    q, sf = oracle.mxfp8(x, order=-1)
    v, s = oracle.mxfp8_decode(q, sf, 64, 256, order=-1)
    recon = (v.reshape(64, 8, 32) * s.reshape(64, 8, 1)).reshape(64, 256)
    # e4m3 keeps 3 mantissa bits: relative error <= 2^-4 below the e4m3 max;
    # scaled values in (448, 512) saturate to 448 (OCP MX clamps), <= 1/8.
    big = np.abs(x) > np.abs(x).max() * 2.0 ** -6
    rel = np.abs(recon - x)[big] / np.abs(x)[big]
    assert rel.max() <= 0.125 + 1e-7
    assert np.median(rel) <= 2.0 ** -4
    # The block amax maps into [256, 512) after scaling by 2^-e.
    amax = np.abs(x.reshape(64, 8, 32)).max(axis=2)
    e = np.floor(np.log2(amax)) - 8
    assert np.array_equal(sf.reshape(64, 8).astype(np.int64), (e + 127).astype(np.int64))


def test_blocks_with_ts_and_linear_to_mma(oracle):
    """O1's block step under a given tensor scale (the tc6 requant rule)
    equals O1 when handed O1's own tensor scale, and the REF_LINEAR -> MMA
    conversion used by the requant parity tests equals the oracle's direct
    MMA quantizer."""
    x = oracle.normal(130 * 64, 5).reshape(130, 64)
    q, sf, ts = oracle.nvfp4_reference(x)
    q2, sf2 = oracle.nvfp4_with_ts(x, ts)
    assert np.array_equal(q, q2) and np.array_equal(sf, sf2)
    for order in (0, 1):
        qm, sm, _ = oracle.nvfp4_mma(x, order)
        a, b = oracle.linear_to_mma(q, sf, 130, 64, order)
        assert np.array_equal(a, qm) and np.array_equal(b, sm)


def test_mxfp4_oracle_known_answers(oracle):
    """OCP MX v1.0 E2M1 rule worked by hand: block amax 1 -> shared exponent
    floor(log2 1) - 2 = -2 (ue8m0 125), elements x * 4 rounded to the e2m1
    grid (ties to even), saturating at 6; an all-zero block gets code 0."""
    x = np.zeros((1, 64), np.float32)
    x[0, :8] = [1.0, 0.5, 0.25, 0.3, -0.0625, 0.8125, -1.0, 0.375]
    q, sf = oracle.mxfp4(x, -1)
    assert sf.tolist() == [125, 0]
    # x*4 = 4, 2, 1, 1.2, -0.25, 3.25, -4, 1.5 -> codes 6, 4, 2, 2, 8 (-0), 5, 14, 3
    codes = [6, 4, 2, 2, 8, 5, 14, 3]
    assert q[:4].tolist() == [(codes[i] << 4) | codes[i + 1] for i in range(0, 8, 2)]
    assert not q[4:].any()
    v, s = oracle.mxfp4_decode(q, sf, 1, 64, -1)
    assert np.allclose(v[:8] * s[0], [1.0, 0.5, 0.25, 0.25, -0.0, 0.75, -1.0, 0.375])
    # MMA order: low nibble first, scales at the L1 offsets
    qm, sm = oracle.mxfp4(x, 0)
    assert qm[0] == (codes[1] << 4) | codes[0]
    assert sm[0] == 125


@pytest.mark.parametrize("rows,k,order", [(300, 512, 0), (300, 512, 1), (128, 64, 0), (1000, 2048, 1)])
def test_row_selected_decode_matches_full_decode(oracle, rows, k, order):
    """The sampled-row views used by the at-scale GPU parity tests
    (scale_rows / nvfp4_rows / mxfp8_rows) equal the full decoders' rows."""
    x = oracle.normal(rows * k, 3).reshape(rows, k)
    idx = sorted({0, 5, 131 % rows, 299 % rows, rows - 1})
    q, sf, _ = oracle.nvfp4_mma(x, order)
    v, s = oracle.nvfp4_decode(q, sf, rows, k, order)
    v2, s2 = oracle.nvfp4_rows(q, sf, idx, rows, k, order)
    assert np.array_equal(v.reshape(rows, k)[idx].ravel(), v2)
    assert np.array_equal(s.reshape(rows, -1)[idx].ravel(), s2)
    q8, sf8 = oracle.mxfp8(x, order)
    v8, s8 = oracle.mxfp8_decode(q8, sf8, rows, k, order)
    v9, s9 = oracle.mxfp8_rows(q8, sf8, idx, rows, k, order)
    assert np.array_equal(v8.reshape(rows, k)[idx].ravel(), v9)
    assert np.array_equal(s8.reshape(rows, -1)[idx].ravel(), s9)
