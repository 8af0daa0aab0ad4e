"""CPU tests of bench.py's host logic: the parity checker it runs in its
cpu_baseline leg must pass a correct sample and flag a wrong quantised byte
or a wrong output, and both arms must emit the same config object."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _sample(oracle, m=256, n=512, k=256):
    xa = oracle.normal(m * k, 5).reshape(m, k)
    xb = oracle.normal(n * k, 6).reshape(n, k)
    qa, sa, ta = oracle.nvfp4_mma(xa, 0)
    qb, sb, tb = oracle.nvfp4_mma(xb, 0)
    rows, cols = bench.sample_rows(m, 16), bench.sample_cols(n, 64)
    av, asf = oracle.nvfp4_rows(qa, sa, rows, m, k, 0)
    bv, bsf = oracle.nvfp4_rows(qb, sb, cols, n, k, 0)
    c = oracle.gemm(av, bv, asf, bsf, len(rows), len(cols), k, 16)
    c = c * np.float32(np.float32(ta) * np.float32(tb))
    # bf16 rounding of the GPU's output (round to nearest even on the top half)
    u = c.astype(np.float32).view(np.uint32)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return {"rows": rows, "cols": cols, "m": m, "n": n, "k": k, "bf16": True,
            "layout_order": 0, "xa_rows": xa[rows], "xb_rows": xb[cols],
            "amax_a": float(np.abs(xa).max()), "amax_b": float(np.abs(xb).max()),
            "ts_a": ta, "ts_b": tb,
            "qa_rows": qa.reshape(m, k // 2)[rows], "sfa": sa,
            "qb_rows": qb.reshape(n, k // 2)[cols], "sfb": sb, "c": u.view(np.float32)}


def test_cpu_check_passes_a_correct_sample(oracle):
    out = bench.cpu_check(_sample(oracle))
    assert out["status"] == "ok" and out["quantizer_bytes"] == "bit-exact", out


def test_cpu_check_flags_a_wrong_quantised_byte(oracle):
    chk = _sample(oracle)
    chk["qb_rows"] = chk["qb_rows"].copy()
    chk["qb_rows"][3, 7] ^= 0x11
    assert bench.cpu_check(chk)["status"] == "FAIL"


def test_cpu_check_flags_a_wrong_output(oracle):
    chk = _sample(oracle)
    chk["c"] = chk["c"].copy()
    chk["c"][2, 10] += 0.5 * np.abs(chk["c"]).max()
    out = bench.cpu_check(chk)
    assert out["status"] == "FAIL" and out["gemm"] == "OUT OF TOLERANCE"


@pytest.mark.parametrize("name", ["colpar", "nvfp4_8192", "skinny_m16"])
@pytest.mark.parametrize("world", [1, 2, 8])
def test_both_arms_emit_the_same_config(name, world):
    w = bench.WORKLOADS[name]
    a = bench.workload_config(name, w, world, 0)
    b = bench.workload_config(name, w, world, 0)
    assert a == b and a["m"] == w["m"] and a["n"] == w["n"]
    if name == "colpar":
        assert a["n_per_rank"] == bench.shard_range(w["n"], world, 0)[1]


def test_shard_range_matches_colpar():
    from cuda_optimazation_b200 import colpar
    for n in (53248, 1000, 28672 + 17):
        for world in (1, 2, 3, 8):
            for r in range(world):
                assert bench.shard_range(n, world, r) == colpar.shard_range(n, world, r)
