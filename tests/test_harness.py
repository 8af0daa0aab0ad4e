"""The drop-in quant_gemm_sm110_bench binary: CLI, CSV contract and exit codes
of GEMMquant_sm110/src/quant_gemm_bench.cu (:3038-3095, :1512-1534) and the
CUTLASS 72b output the sweep runner parses
(GEMMquant_sm110/scripts/run_quant_gemm_1024.py:404-410)."""
import csv
import re
import subprocess

import pytest

HEADER = ["BackendId", "Version", "N", "Precision", "Reference", "TimeMs", "GFLOPS",
          "RatioToReference", "Matched"]


@pytest.fixture(scope="module")
def binary(qlib):
    from cuda_optimazation_b200 import build
    return build.build_harness()


def test_bad_arguments_exit_nonzero(binary):
    r = subprocess.run([str(binary), "256", "no_such_backend"], capture_output=True, text=True)
    assert r.returncode != 0 and "Usage" in r.stderr


def test_multi_gpu_only_for_colpar(binary):
    r = subprocess.run([str(binary), "512", "512", "512", "nvfp4_q1_native_fp4_mainloop",
                        "--gpus", "2"], capture_output=True, text=True)
    assert r.returncode != 0 and "only nvfp4_colpar_q0" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("args", [["256", "all"], ["1024", "all"],
                                  ["512", "1024", "768", "nvfp4_q1_native_fp4_mainloop",
                                   "--out-dtype", "bf16"],
                                  ["64", "4096", "2048", "nvfp4_skinny_q0", "--gpus", "1",
                                   "--dist", "normal", "--seed", "7"],
                                  ["512", "768", "1024", "nvfp4_q0_tc6_fused_epilogue"],
                                  ["384", "640", "1024", "mxfp4_q0_tcgen05_block_scaled",
                                   "--out-dtype", "bf16"]])
def test_csv_rows_matched(binary, tmp_path, args):
    r = subprocess.run([str(binary), *args], capture_output=True, text=True, cwd=tmp_path,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    rows = list(csv.DictReader(open(tmp_path / "quant_sm110_benchmark.csv")))
    with open(tmp_path / "quant_sm110_benchmark.csv") as f:
        assert f.readline().strip().split(",")[:9] == HEADER
    assert rows and all(row["Matched"] == "1" for row in rows)
    assert all(float(row["GFLOPS"]) > 0 for row in rows)
    # Rates relative to the cuBLASLt FP8 GEMM timed in the same run.
    assert all(float(row["RatioToReference"]) > 0 for row in rows)
    assert re.search(r"backend_id=\S+ time_ms=\S+ work_unit=flop rate_per_second=\S+ "
                     r"reference_rate_per_second=\S+ matched=1", r.stdout)


@pytest.mark.gpu
def test_cutlass_cli_form(binary, tmp_path):
    r = subprocess.run([str(binary), "--m=1024", "--n=1024", "--k=1024", "--iterations=20",
                        "--swizzle=2"], capture_output=True, text=True, cwd=tmp_path, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    # parse_cutlass_fp4_stdout
    assert "Disposition: Passed" in r.stdout
    t = re.search(r"Avg runtime:\s*([0-9.eE+-]+)\s*ms", r.stdout)
    g = re.search(r"GFLOPS:\s*([0-9.eE+-]+)", r.stdout)
    assert t and g and float(t.group(1)) > 0 and float(g.group(1)) > 0


@pytest.mark.gpu
def test_cutlass_cli_form_mxfp4_name(binary, tmp_path):
    """Under the MXFP4 runner's binary name the CUTLASS CLI runs MXFP4
    (run_quant_gemm_1024.py --cutlass-mxfp4-bin, :615-624)."""
    mx = binary.parent / "cutlass_72a_mxfp4_bf16_b200"
    r = subprocess.run([str(mx), "--m=512", "--n=512", "--k=1024", "--iterations=10",
                        "--swizzle=1"], capture_output=True, text=True, cwd=tmp_path, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Backend: mxfp4_q0_tcgen05_block_scaled" in r.stdout
    assert "Disposition: Passed" in r.stdout


def test_option_validation_without_gpu(binary):
    """--dist accepts only the harness's normal law and --gpus only 1 (the
    multi-GPU split is the column-parallel bench); both fail before any GPU
    call."""
    for extra in (["--dist", "uniform"], ["--gpus", "8"]):
        r = subprocess.run([str(binary), "256", "256", "256", "nvfp4_q1_native_fp4_mainloop",
                            *extra], capture_output=True, text=True, timeout=60)
        assert r.returncode != 0 and "Usage" in r.stderr


def _colpar_run(binary, tmp_path, gpus):
    r = subprocess.run([str(binary), "1024", "2560", "1024", "nvfp4_colpar_q0", "--gpus",
                        str(gpus), "--out-dtype", "bf16"], capture_output=True, text=True,
                       cwd=tmp_path, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    rows = list(csv.DictReader(open(tmp_path / "quant_sm110_benchmark.csv")))
    assert [row["BackendId"] for row in rows] == ["nvfp4_colpar_q0"]
    assert rows[0]["Matched"] == "1" and rows[0]["GPUs"] == str(gpus)
    assert "GEMM only" in r.stdout


@pytest.mark.gpu
def test_colpar_backend_one_gpu(binary, tmp_path):
    """The column-parallel backend on one GPU: the gather degenerates to the
    GPU's own C; the check runs on that full C."""
    _colpar_run(binary, tmp_path, 1)


@pytest.mark.gpu
@pytest.mark.skipif(__import__("torch").cuda.device_count() < 2, reason="needs 2 GPUs")
def test_colpar_backend_two_gpus(binary, tmp_path):
    """B split along N over two GPUs of one process; every GPU's epilogue
    stores its columns into both GPUs' C over NVLink; both Cs are checked."""
    _colpar_run(binary, tmp_path, 2)


@pytest.mark.gpu
def test_cublaslt_nvfp4_library_row(binary, tmp_path):
    """The vendor library's NVFP4 GEMM over this library's quantised bytes
    (K-major scale tiles) passes the same oracle check: the same-box
    comparison row for the FP4 backend."""
    r = subprocess.run([str(binary), "1024", "1536", "2048", "cublaslt_nvfp4_library"],
                       capture_output=True, text=True, cwd=tmp_path, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    rows = list(csv.DictReader(open(tmp_path / "quant_sm110_benchmark.csv")))
    assert rows[0]["BackendId"] == "cublaslt_nvfp4_library" and rows[0]["Matched"] == "1"
