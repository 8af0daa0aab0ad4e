"""GPU: a qg_plan (host work of a GEMM call done once) gives the same bytes
as the direct entry point in every format, reads the operands at run time,
and runs repeatedly."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp8", "mxfp4"])
@pytest.mark.parametrize("m,n,k", [(256, 512, 512), (100, 256, 256)])
def test_plan_matches_direct_call(qlib, fmt, m, n, k):
    make = {"nvfp4": qlib.make_nvfp4, "mxfp8": qlib.make_mxfp8, "mxfp4": qlib.make_mxfp4}[fmt]
    g = torch.Generator(device="cuda").manual_seed(5)
    xa = torch.randn(m, k, generator=g, device="cuda")
    xb = torch.randn(n, k, generator=g, device="cuda")
    A, B = make(xa), make(xb)
    direct = qlib.block_scaled_gemm(A, B, torch.bfloat16)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    with qlib.GemmPlan(A, B, out) as plan:
        got = plan.run()
        torch.cuda.synchronize()
        assert torch.equal(got, direct)
        # New operand contents in the same buffers: the plan reads them at run time.
        A2 = make(xa * 0.5)
        A.quantized.copy_(A2.quantized)
        A.block_scales.copy_(A2.block_scales)
        if fmt == "nvfp4":
            A.tensor_scale.copy_(A2.tensor_scale)
        plan.run()
        plan.run()
        torch.cuda.synchronize()
        assert torch.equal(out, qlib.block_scaled_gemm(A2, B, torch.bfloat16))
