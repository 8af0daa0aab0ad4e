"""Build the sm_100a shared library in-tree.

    python -m cuda_optimazation_b200.build

Compiles every .cu under csrc/ with nvcc for sm_100a only and links
cuda_optimazation_b200/libqgemm_b200.so (C ABI: include/qgemm.h).  The
library resolves cuTensorMapEncodeTiled through the CUDA runtime's driver
entry point, so it needs no libcuda at link time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "libqgemm_b200.so"
OBJ = PKG / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-Xptxas", "-v",
    f"-I{ROOT / 'include'}",
] + os.environ.get("QG_EXTRA_NVCC", "").split()


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(CSRC.glob("*")) + [ROOT / "include" / "qgemm.h", Path(__file__), HARNESS_SRC]
    if not HARNESS_BIN.exists():
        return True
    return any(d.stat().st_mtime > t for d in deps if d.is_file())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return OUT
    OBJ.mkdir(exist_ok=True)
    from concurrent.futures import ThreadPoolExecutor

    def compile_one(src: Path) -> str:
        obj = OBJ / (src.stem + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        (OBJ / (src.stem + ".ptxas.txt")).write_text(r.stdout + r.stderr)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"nvcc failed on {src.name}")
        if verbose:
            sys.stdout.write(r.stderr)
        return str(obj)

    # One nvcc per translation unit, in parallel (each is single-threaded).
    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp),
           *objs, "-lcudart_static", "-lrt", "-lpthread", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link failed")
    os.replace(tmp, OUT)
    build_harness()
    return OUT


HARNESS_SRC = PKG / "harness" / "quant_gemm_bench.cpp"
HARNESS_BIN = PKG / "bin" / "quant_gemm_sm110_bench"
HARNESS_MXFP4_BIN = PKG / "bin" / "cutlass_72a_mxfp4_bf16_b200"


def build_harness() -> Path:
    """The drop-in quant_gemm_sm110_bench binary, linked against the library
    (rpath $ORIGIN/..)."""
    HARNESS_BIN.parent.mkdir(exist_ok=True)
    cmd = [nvcc(), "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
           f"-I{ROOT / 'include'}", str(HARNESS_SRC), "-o", str(HARNESS_BIN),
           f"-L{PKG}", "-lqgemm_b200", "-lcublasLt", "-Xlinker", "-rpath=$ORIGIN/.."]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("harness build failed")
    # The same binary under the MXFP4 runner's name: its --m/--n/--k form
    # then runs MXFP4 (what run_quant_gemm_1024.py's --cutlass-mxfp4-bin
    # points at).
    shutil.copy2(HARNESS_BIN, HARNESS_MXFP4_BIN)
    return HARNESS_BIN


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(OUT)
