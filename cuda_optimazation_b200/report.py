"""Sweep and report: the reference's reporting step for the quant-GEMM path.

The reference's sweep runner (GEMMquant_sm110/scripts/run_quant_gemm_1024.py)
runs each backend binary per trial and writes one CSV row per (backend,
trial) with the header CSV_HEADER; its plotter
(GEMMquant_sm110/scripts/plot_quant_gemm.py) reads that CSV (rows with
Status == "ok" and Matched == "1") and draws the best backend per precision.

    python -m cuda_optimazation_b200.report sweep --n 8192 --trials 3 --out sweep.csv
        runs this library's drop-in harness (quant_gemm_sm110_bench) for every
        B200 backend and writes the runner's CSV, so the reference's
        plot_quant_gemm.py plots it unchanged.  RatioToReference is taken
        against a cuBLAS bf16 GEMM of the same size timed in the same run (the
        reference's ratios are against cuBLAS tensor-core GEMMs).
    python -m cuda_optimazation_b200.report roofline --csv quant_sm110_benchmark.csv \\
        --out roofline.svg [--peaks MEASURED_PEAKS.json]
        draws a B200 roofline (measured HBM and tensor-core roofs) with every
        matched harness row placed by its arithmetic intensity.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import subprocess
import tempfile
from html import escape
from pathlib import Path
from typing import Optional

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent

# The sweep runner's CSV header (run_quant_gemm_1024.py:9-23).
CSV_HEADER = ["Precision", "Stage", "BackendId", "BackendLabel", "N", "Reference", "TimeMs",
              "GFLOPS", "RatioToReference", "Matched", "Status", "Reason", "Trial"]

# Backends of the drop-in harness, in the runner's (precision, stage) slots.
BACKENDS = [
    dict(precision="NVFP4", stage="q0", backend_id="nvfp4_q0_tc6_fused_epilogue",
         label="B200 tcgen05 NVFP4 GEMM, NVFP4 output requantised in the epilogue"),
    dict(precision="NVFP4", stage="q1", backend_id="nvfp4_q1_native_fp4_mainloop",
         label="B200 tcgen05 kind::mxf4nvf4 CTA-pair NVFP4 GEMM (bf16 out)", bf16=True),
    dict(precision="MXFP4", stage="q0", backend_id="mxfp4_q0_tcgen05_block_scaled",
         label="B200 tcgen05 kind::mxf4nvf4.block32 MXFP4 GEMM (bf16 out)", bf16=True),
    dict(precision="FP8", stage="q0", backend_id="mxfp8_q0_tcgen05_block_scaled",
         label="B200 tcgen05 kind::mxf8f6f4 MXFP8 GEMM (bf16 out)", bf16=True),
]

# Dense tensor-core rate of each format relative to bf16 on B200.
_RATE_VS_BF16 = {"nvfp4": 4.0, "mxfp4": 4.0, "mxfp8": 2.0}
_NOMINAL = {"hbm_gbs": 7700.0, "bf16_tflops": 2250.0}


def harness_binary() -> Path:
    return PKG / "bin" / "quant_gemm_sm110_bench"


def cublas_bf16_gflops(n: int, reps: int = 20) -> float:
    """cuBLAS bf16 GEMM rate at n^3 (torch.matmul), CUDA-event timed."""
    import torch
    a = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(n, n, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        torch.matmul(a, b)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        torch.matmul(a, b)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return 2.0 * n ** 3 / (ms * 1e6)


def _harness_row(stdout_csv: Path, backend_id: str) -> Optional[dict]:
    if not stdout_csv.exists():
        return None
    with stdout_csv.open(newline="") as f:
        for row in csv.DictReader(f):
            if row.get("BackendId") == backend_id:
                return row
    return None


def sweep(n: int, trials: int, out: Path, binary: Optional[Path] = None,
          reference_gflops: Optional[float] = None, timeout: int = 600) -> list[dict]:
    """Run every backend `trials` times at n^3 and write the runner's CSV."""
    binary = binary or harness_binary()
    if reference_gflops is None:
        reference_gflops = cublas_bf16_gflops(n)
    rows = []
    for trial in range(trials):
        for b in BACKENDS:
            with tempfile.TemporaryDirectory() as d:
                args = [str(binary), str(n), str(n), str(n), b["backend_id"]]
                if b.get("bf16"):
                    args += ["--out-dtype", "bf16"]
                proc = subprocess.run(args, cwd=d, capture_output=True, text=True,
                                      timeout=timeout)
                src = _harness_row(Path(d) / "quant_sm110_benchmark.csv", b["backend_id"])
            base = {"Precision": b["precision"], "Stage": b["stage"],
                    "BackendId": b["backend_id"], "BackendLabel": b["label"], "N": str(n),
                    "Reference": "cuBLAS bf16 tensor-core GEMM (torch.matmul)",
                    "Trial": str(trial)}
            if proc.returncode != 0 or src is None:
                reason = f"harness exited with status {proc.returncode}"
                rows.append(dict(base, TimeMs="", GFLOPS="", RatioToReference="", Matched="0",
                                 Status="missing" if src is None else "failed", Reason=reason))
                continue
            gflops = float(src["GFLOPS"])
            matched = src.get("Matched", "0")
            rows.append(dict(base, TimeMs=src["TimeMs"], GFLOPS=src["GFLOPS"],
                             RatioToReference=f"{gflops / reference_gflops:.6g}",
                             Matched=matched, Status="ok" if matched == "1" else "failed",
                             Reason="" if matched == "1" else "harness check failed"))
    with out.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=CSV_HEADER)
        w.writeheader()
        w.writerows(rows)
    return rows


# ----------------------------------------------------------------- roofline
def _format_of(precision: str) -> Optional[str]:
    p = precision.lower()
    for fmt in ("nvfp4", "mxfp4", "mxfp8"):
        if p.startswith(fmt):
            return fmt
    return None


def algorithmic_bytes(fmt: str, out: str, m: int, n: int, k: int) -> float:
    """Operand + scale bytes read and output bytes written once per GEMM."""
    if fmt == "nvfp4":
        per_elem = 0.5 + 1.0 / 16
    elif fmt == "mxfp4":
        per_elem = 0.5 + 1.0 / 32
    else:
        per_elem = 1.0 + 1.0 / 32
    out_bytes = {"bf16": 2.0, "fp32": 4.0, "nvfp4": 0.5 + 1.0 / 16}.get(out, 2.0)
    return (m + n) * k * per_elem + m * n * out_bytes


def harness_points(csv_path: Path) -> list[dict]:
    """Matched rows of a harness CSV (quant_sm110_benchmark.csv) as
    (label, format, intensity FLOP/B, TFLOP/s) points."""
    pts = []
    with csv_path.open(newline="") as f:
        for row in csv.DictReader(f):
            if row.get("Matched") != "1":
                continue
            fmt = _format_of(row.get("Precision", ""))
            if fmt is None:
                continue
            m = int(row.get("M") or row["N"])
            n = int(row.get("NCols") or row["N"])
            k = int(row.get("K") or row["N"])
            out = row["Precision"].split("->")[-1]
            flops = 2.0 * m * n * k
            tflops = float(row["GFLOPS"]) / 1e3
            pts.append(dict(label=f"{row['BackendId']} {m}x{n}x{k}", fmt=fmt,
                            intensity=flops / algorithmic_bytes(fmt, out, m, n, k),
                            tflops=tflops))
    return pts


def load_peaks(path: Optional[Path]) -> dict:
    if path and path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    return dict(_NOMINAL, source="nominal")


def roofline_svg(points: list[dict], peaks: dict, width: int = 900, height: int = 560) -> str:
    """A log-log roofline: HBM roof and one tensor roof per format, points
    placed by arithmetic intensity and achieved TFLOP/s."""
    left, right, top, bottom = 80, 220, 40, 60
    pw, ph = width - left - right, height - top - bottom
    x0, x1 = 1.0, 1e5                 # FLOP per byte
    roofs = {fmt: peaks["bf16_tflops"] * r for fmt, r in _RATE_VS_BF16.items()}
    y0, y1 = 10.0, 10 ** math.ceil(math.log10(max(roofs.values()) * 1.5))
    hbm_tbs = peaks["hbm_gbs"] / 1e3

    def px(x):
        return left + pw * (math.log10(x) - math.log10(x0)) / (math.log10(x1) - math.log10(x0))

    def py(y):
        return top + ph * (1 - (math.log10(y) - math.log10(y0)) / (math.log10(y1) - math.log10(y0)))

    colors = {"nvfp4": "#2563eb", "mxfp4": "#16a34a", "mxfp8": "#dc2626"}
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" '
           f'font-family="sans-serif" font-size="12">',
           f'<rect x="0" y="0" width="{width}" height="{height}" fill="white"/>',
           f'<text x="{left}" y="22" font-size="15">B200 roofline ({escape(peaks["source"])} '
           f'peaks: HBM {peaks["hbm_gbs"]:.0f} GB/s, bf16 {peaks["bf16_tflops"]:.0f} TF/s)</text>',
           f'<rect x="{left}" y="{top}" width="{pw}" height="{ph}" fill="none" stroke="#888"/>']
    for e in range(int(math.log10(x0)), int(math.log10(x1)) + 1):
        x = px(10 ** e)
        out.append(f'<line x1="{x:.1f}" y1="{top}" x2="{x:.1f}" y2="{top + ph}" stroke="#eee"/>')
        out.append(f'<text x="{x:.1f}" y="{top + ph + 16}" text-anchor="middle">1e{e}</text>')
    for e in range(int(math.log10(y0)), int(math.log10(y1)) + 1):
        y = py(10 ** e)
        out.append(f'<line x1="{left}" y1="{y:.1f}" x2="{left + pw}" y2="{y:.1f}" stroke="#eee"/>')
        out.append(f'<text x="{left - 6}" y="{y + 4:.1f}" text-anchor="end">1e{e}</text>')
    out.append(f'<text x="{left + pw / 2}" y="{height - 14}" text-anchor="middle">'
               f'arithmetic intensity (FLOP / algorithmic byte)</text>')
    out.append(f'<text x="18" y="{top + ph / 2}" transform="rotate(-90 18 {top + ph / 2})" '
               f'text-anchor="middle">TFLOP/s</text>')
    for fmt, roof in roofs.items():
        ridge = roof / hbm_tbs
        pts = [(x0, hbm_tbs * x0), (ridge, roof), (x1, roof)]
        path = " ".join(f"{px(a):.1f},{py(max(b, y0)):.1f}" for a, b in pts)
        out.append(f'<polyline points="{path}" fill="none" stroke="{colors[fmt]}" '
                   f'stroke-width="1.5" stroke-dasharray="6,3"/>')
        out.append(f'<text x="{left + pw + 6}" y="{py(roof) + 4:.1f}" fill="{colors[fmt]}">'
                   f'{fmt} roof {roof:.0f} TF/s</text>')
    for i, p in enumerate(points):
        x, y = px(min(max(p["intensity"], x0), x1)), py(min(max(p["tflops"], y0), y1))
        c = colors.get(p["fmt"], "#333")
        out.append(f'<circle cx="{x:.1f}" cy="{y:.1f}" r="4" fill="{c}"><title>'
                   f'{escape(p["label"])}: {p["tflops"]:.0f} TF/s</title></circle>')
        out.append(f'<text x="{left + pw + 6}" y="{top + 90 + 14 * i}" fill="{c}">'
                   f'{escape(p["label"][:28])} {p["tflops"]:.0f}</text>')
    out.append("</svg>")
    return "\n".join(out)


def main(argv: Optional[list[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m cuda_optimazation_b200.report")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("sweep", help="run every backend, write the sweep runner's CSV")
    s.add_argument("--n", type=int, default=8192)
    s.add_argument("--trials", type=int, default=3)
    s.add_argument("--out", type=Path, default=Path("quant_gemm_b200_sweep.csv"))
    r = sub.add_parser("roofline", help="B200 roofline SVG from a harness CSV")
    r.add_argument("--csv", type=Path, required=True)
    r.add_argument("--out", type=Path, required=True)
    r.add_argument("--peaks", type=Path, default=ROOT / "MEASURED_PEAKS.json")
    a = ap.parse_args(argv)
    if a.cmd == "sweep":
        rows = sweep(a.n, a.trials, a.out)
        bad = [x for x in rows if x["Status"] != "ok"]
        print(f"wrote {a.out}: {len(rows)} rows, {len(bad)} not ok")
        return 1 if bad else 0
    pts = harness_points(a.csv)
    a.out.write_text(roofline_svg(pts, load_peaks(a.peaks)))
    print(f"wrote {a.out}: {len(pts)} points")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
