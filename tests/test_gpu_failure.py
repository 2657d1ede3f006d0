"""The bounded-wait failure path on the GPU, without a fault: a kernel waits
on an mbarrier nothing arrives on, through the same bounded wait every
waiting kernel of the library uses. The wait gives up at its limit, the
status word reads D3_STATUS_WAIT_TIMEOUT, and the context keeps working."""

from __future__ import annotations

import time

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_wait_gives_up_and_reports_in_the_status_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import _lib
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.monotonic()
    _lib.call("d3_wait_timeout_probe", status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert int(status.item()) == _lib.D3_STATUS_WAIT_TIMEOUT
    assert 1.0 < waited < 30.0  # the 2 s limit, not an open-ended spin
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum().item()) == 56.0  # the context is still usable
