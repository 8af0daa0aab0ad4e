"""qg_quantize_nvfp4_noalloc: the NVFP4 quantizer entry point for callers that
cannot allocate device memory (framework-hosted plugins that only see the
call's tensors, allocator-free runtimes, code inside allocator callbacks,
loops that cannot take cudaMalloc's implicit synchronisation).  It keeps its
amax scratch in a fixed array inside the library instead of a caller
workspace.  Checked through the C ABI against qg_quantize_nvfp4 on two calls
in a row; the outputs are integer codes, so the tolerance is bit equality.
This file sorts last so a run that stops at the first failure has already run
every other test."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _quantize_both(L, x, layout):
    rows, k = x.shape
    dev = x.device
    n = rows * k
    nb = (n + 15) // 16
    nsf = nb if layout == 0 else int(L.qg_scale_bytes(rows, k, 16))
    outs = []
    for noalloc in (False, True):
        q = torch.full((nb * 8,), 0xAA, dtype=torch.uint8, device=dev)
        sf = torch.full((nsf,), 0xAA, dtype=torch.uint8, device=dev)
        ts = torch.full((1,), -1.0, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream().cuda_stream
        dt = 1 if x.dtype == torch.bfloat16 else 0
        if noalloc:
            rc = L.qg_quantize_nvfp4_noalloc(x.data_ptr(), dt, rows, k, layout, q.data_ptr(),
                                             sf.data_ptr(), ts.data_ptr(), stream)
        else:
            ws = torch.empty(int(L.qg_quantize_workspace_bytes()), dtype=torch.uint8, device=dev)
            rc = L.qg_quantize_nvfp4(x.data_ptr(), dt, rows, k, layout, q.data_ptr(),
                                     sf.data_ptr(), ts.data_ptr(), ws.data_ptr(), stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        outs.append((q.cpu().numpy(), sf.cpu().numpy(), float(ts.item())))
    return outs


@pytest.mark.parametrize("layout", [0, 1])
def test_noalloc_matches_workspace_entry_point_twice(qlib, layout):
    L = qlib.lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    # Two calls in a row with different inputs: the second must not see the
    # first call's scratch contents.
    x1 = torch.randn(1024, 2048, generator=g, device="cuda") * 3.0
    x2 = torch.randn(384, 4096, generator=g, device="cuda").to(torch.bfloat16)
    for x in (x1, x2):
        (qa, sa, ta), (qb, sb, tb) = _quantize_both(L, x, layout)
        assert ta == tb
        assert np.array_equal(qa, qb)
        assert np.array_equal(sa, sb)


def test_noalloc_rejects_inputs_over_capacity(qlib):
    L = qlib.lib()
    cap = int(L.qg_quantize_nvfp4_noalloc_max_elements())
    assert cap == 1 << 28
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    rc = L.qg_quantize_nvfp4_noalloc(dummy.data_ptr(), 0, cap // 1024 + 1, 1024, 1,
                                     dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == qlib.ERR_SHAPE


@pytest.mark.parametrize("rows,k,layout", [
    (3, 1001, 0),            # REF_LINEAR, rows*k not a multiple of 16 (zero-padded last block)
    (7, 16384 * 5 + 48, 0),  # the last amax slot covers a partial 16384-element chunk
    (130, 1040, 1),          # MMA layout with padded scale rows and columns
])
def test_noalloc_ragged_sizes(qlib, rows, k, layout):
    L = qlib.lib()
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + k)
    x = torch.randn(rows, k, generator=g, device="cuda")
    (qa, sa, ta), (qb, sb, tb) = _quantize_both(L, x, layout)
    assert ta == tb
    assert np.array_equal(qa, qb) and np.array_equal(sa, sb)


@pytest.mark.parametrize("specials", [("inf",), ("-inf",), ("nan",), ("nan", "inf", "-inf")])
def test_noalloc_special_values(qlib, specials):
    """+-inf and NaN inputs: both entry points reduce the amax the same way
    (NaN ignored, as std::max in the reference quantizer does) and write the
    same bytes."""
    L = qlib.lib()
    g = torch.Generator(device="cuda").manual_seed(11)
    for dtype in (torch.float32, torch.bfloat16):
        x = torch.randn(64, 512, generator=g, device="cuda")
        for i, sv in enumerate(specials):
            x.view(-1)[1000 * i + 37] = float(sv)
        x = x.to(dtype)
        (qa, sa, ta), (qb, sb, tb) = _quantize_both(L, x, 0)
        assert ta == tb or (np.isnan(ta) and np.isnan(tb))
        assert np.array_equal(qa, qb) and np.array_equal(sa, sb)
