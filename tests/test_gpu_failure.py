"""Failure detection on the device without a GPU fault.

Every kernel that waits on an mbarrier gives up after a bounded time, records
a code in its device error flag and unwinds; the host reports
CLEF_ERR_DEVICE_TIMEOUT. clef_selftest_wait_timeout runs exactly that path on
a barrier nothing arrives on, with a short limit: the call must come back with
the timeout status after about the limit (not hang), and the CUDA context must
stay usable for the next kernel.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("limit_ms", [50, 300])
def test_stuck_wait_ends_as_a_status_and_the_context_survives(limit_ms):
    import clef_b200 as cb
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = cb.lib.clef_selftest_wait_timeout(limit_ms, None)
    elapsed = time.perf_counter() - t0
    assert rc == 6, cb.lib.clef_last_error().decode()
    assert "gave up" in cb.lib.clef_last_error().decode()
    assert limit_ms / 1000 <= elapsed < limit_ms / 1000 + 5.0
    # The context is intact: a kernel launched afterwards runs and is correct.
    x = torch.randn(37, 2560, device="cuda")
    w = torch.rand(2560, device="cuda")
    y = cb.rmsnorm(x, w, eps=1e-6, out_dtype=cb.F32)
    ref = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6) * w
    assert float((y - ref).abs().max()) <= 1e-5
