"""Bounded-wait failure path on the GPU: a wait nothing satisfies must end
with QG_ERR_TIMEOUT in a short time and leave the context usable."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_timeout_reports_status(qlib):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    qlib.selftest_wait_timeout(50_000_000, status)  # 50 ms bound
    rc, code = qlib.read_status(status)
    assert rc == qlib.ERR_TIMEOUT and code == 4
    assert time.time() - t0 < 5.0
    # Context still healthy afterwards.
    x = torch.ones(1024, device="cuda")
    assert float(x.sum().item()) == 1024.0
    rc, code = qlib.read_status(status)
    assert rc == qlib.OK and code == 0


def test_selftest_rejects_long_bounds(qlib):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(qlib.QGemmError):
        qlib.selftest_wait_timeout(10_000_000_000, status)
