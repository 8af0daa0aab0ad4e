"""Generate the golden fixtures in this folder from the REFERENCE's own code.

Runs oracle/_ref/libqg_ref.so, which is the reference's host headers
(GEMMsm110/include/requant/nvfp4_reference.cuh, cutlass-gemm-cpp-guide/
include/guide/block_scale_reference.hpp) compiled behind oracle/ref_shim.cpp.
Needs the reference checkout (this container only); the fixtures it writes
travel with the repo so tests on machines without the reference can use them.

    python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import oracle as om  # noqa: E402


def main() -> None:
    o, ref = om.Oracle(), om.Reference()
    out = {}
    for dist in om.DISTRIBUTIONS:
        # Inputs: the six distributions of requant_epilogue_benchmark.cu:135-165
        # (std::mt19937 seed 1234), 64 x 64.
        x = o.requant_dist(64 * 64, dist, 1234)
        q, sf, ts = ref.nvfp4_reference(x)
        out[f"{dist}_x"] = x
        out[f"{dist}_q"] = q
        out[f"{dist}_sf"] = sf
        out[f"{dist}_ts"] = np.array([ts], np.float32)
    np.savez_compressed(HERE / "nvfp4_requant_64x64.npz", **out)

    # Block-scaled GEMM: seeded N(0,1) operands quantised to NVFP4 by the
    # reference quantizer, decoded to logical fp32, multiplied by the
    # reference O2 (double accumulation).
    m, n, k = 48, 40, 256
    xa = o.normal(m * k, 20260817)
    xb = o.normal(n * k, 20260817 ^ 0xBB67AE85)
    def logical(xv, rows):
        q, sf, ts = ref.nvfp4_reference(xv)
        lo = q & 0xF
        hi = q >> 4
        codes = np.stack([hi, lo], axis=1).ravel()  # high nibble = first value
        mag = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float32)
        vals = np.where(codes & 8, -mag[codes & 7], mag[codes & 7]).astype(np.float32)
        scales = np.array([ref.L.qgr_decode_e4m3_positive(int(s)) for s in sf], np.float32)
        return vals, scales, ts
    av, asf, ats = logical(xa, m)
    bv, bsf, bts = logical(xb, n)
    d = ref.gemm(av, bv, asf, bsf, m, n, k, 16)
    np.savez_compressed(HERE / "block_scaled_gemm_48x40x256.npz", a=av, b=bv, sfa=asf, sfb=bsf,
                        d=d, ts=np.array([ats, bts], np.float32))
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
