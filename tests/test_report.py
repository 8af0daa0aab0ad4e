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
