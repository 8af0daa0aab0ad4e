"""Reporting step (cuda_optimazation_b200/report.py): the sweep CSV keeps the
reference sweep runner's header (GEMMquant_sm110/scripts/run_quant_gemm_1024.py:9-23)
so its plot_quant_gemm.py reads it, and the roofline SVG places harness rows
by arithmetic intensity under the measured roofs."""
import csv
import xml.etree.ElementTree as ET

import pytest

from cuda_optimazation_b200 import report

RUNNER_HEADER = ["Precision", "Stage", "BackendId", "BackendLabel", "N", "Reference", "TimeMs",
                 "GFLOPS", "RatioToReference", "Matched", "Status", "Reason", "Trial"]


def test_header_and_backends():
    assert report.CSV_HEADER == RUNNER_HEADER
    ids = [b["backend_id"] for b in report.BACKENDS]
    assert "nvfp4_q0_tc6_fused_epilogue" in ids and "nvfp4_q1_native_fp4_mainloop" in ids


def test_roofline_svg(tmp_path):
    p = tmp_path / "h.csv"
    with p.open("w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["BackendId", "Version", "N", "Precision", "Reference", "TimeMs", "GFLOPS",
                    "RatioToReference", "Matched", "TFLOPS", "PctPeak", "GPUs", "M", "NCols", "K"])
        w.writerow(["nvfp4_q1_native_fp4_mainloop", "v", 8192, "nvfp4->bf16", "r", 0.23,
                    4.7e6, 0, 1, 4700, 52, 1, 8192, 8192, 8192])
        w.writerow(["mxfp8_q0_tcgen05_block_scaled", "v", 4096, "mxfp8->bf16", "r", 0.2,
                    2.3e6, 0, 1, 2300, 51, 1, 4096, 14336, 4096])
        w.writerow(["nvfp4_skinny_q0", "v", 16, "nvfp4->bf16", "r", 0.03,
                    2.0e5, 0, 1, 200, 2, 1, 16, 28672, 8192])
        w.writerow(["broken", "v", 16, "nvfp4->bf16", "r", 0.03, 1, 0, 0, 0, 0, 1, 16, 16, 16])
    pts = report.harness_points(p)
    assert len(pts) == 3  # unmatched row dropped
    # NVFP4 8192^3 bf16 out: 2*8192^3 / (2*8192^2*0.5625 + 8192^2*2)
    assert abs(pts[0]["intensity"] - 2 * 8192 / (2 * 0.5625 + 2)) < 1e-6
    assert pts[2]["intensity"] < 100  # decode shape sits left of the ridge
    svg = report.roofline_svg(pts, {"hbm_gbs": 6549.1, "bf16_tflops": 1672.2,
                                    "source": "measured"})
    root = ET.fromstring(svg)
    circles = [e for e in root.iter() if e.tag.endswith("circle")]
    assert len(circles) == 3
    out = tmp_path / "r.svg"
    assert report.main(["roofline", "--csv", str(p), "--out", str(out),
                        "--peaks", str(tmp_path / "none.json")]) == 0
    ET.parse(out)


@pytest.mark.gpu
def test_sweep_small(qlib, tmp_path):
    out = tmp_path / "s.csv"
    rows = report.sweep(512, 1, out)
    assert len(rows) == len(report.BACKENDS)
    assert all(r["Status"] == "ok" and r["Matched"] == "1" for r in rows), rows
    with out.open() as f:
        assert f.readline().strip().split(",") == RUNNER_HEADER


def test_sweep_rows_from_a_stand_in_harness(tmp_path):
    """The sweep's row assembly on CPU: a stand-in harness writes the
    harness CSV (or fails for one backend); rows carry the runner's header,
    Status ok / failed, and the rate ratio to the given reference."""
    fake = tmp_path / "fake_bench"
    fake.write_text(
        "#!/usr/bin/env python3\n"
        "import sys\n"
        "b = sys.argv[4]\n"
        "if b.startswith('mxfp8'):\n"
        "    sys.exit(3)\n"
        "open('quant_sm110_benchmark.csv', 'w').write(\n"
        "    'BackendId,Version,N,Precision,Reference,TimeMs,GFLOPS,RatioToReference,Matched\\n'\n"
        "    f'{b},v,{sys.argv[1]},nvfp4->bf16,r,0.5,2000,0,1\\n')\n")
    fake.chmod(0o755)
    out = tmp_path / "sweep.csv"
    rows = report.sweep(256, 2, out, binary=fake, reference_gflops=1000.0)
    assert len(rows) == 2 * len(report.BACKENDS)
    with out.open() as f:
        got = list(csv.DictReader(f))
    assert list(got[0].keys()) == RUNNER_HEADER
    ok = [r for r in got if r["Status"] == "ok"]
    bad = [r for r in got if r["Status"] != "ok"]
    assert {r["BackendId"] for r in bad} == {"mxfp8_q0_tcgen05_block_scaled"}
    assert all(r["Matched"] == "0" and r["Reason"] for r in bad)
    assert all(float(r["RatioToReference"]) == 2.0 and r["Matched"] == "1" for r in ok)
    assert {r["Trial"] for r in got} == {"0", "1"}
