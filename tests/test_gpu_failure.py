"""The bounded-wait failure path on the GPU, without a fault: a kernel waits
on an mbarrier nothing arrives on, through the same bounded wait every
waiting kernel of the library uses. The wait gives up at its limit, the
status word reads D3_STATUS_WAIT_TIMEOUT, and the context keeps working.
The probe lives in the test-only library libd3moe_selftest.so."""

from __future__ import annotations

import ctypes
import time

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _selftest_lib():
    from d3moe import _lib
    lib = ctypes.CDLL(str(_lib.SELFTEST_LIB_PATH))
    lib.d3_wait_timeout_probe.restype = ctypes.c_int
    lib.d3_wait_timeout_probe.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    return lib


def test_wait_gives_up_and_reports_in_the_status_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import _lib
    _lib.load()
    lib = _selftest_lib()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.monotonic()
    rc = lib.d3_wait_timeout_probe(status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.D3_OK
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert int(status.item()) == _lib.D3_STATUS_WAIT_TIMEOUT
    assert 1.0 < waited < 30.0  # the 2 s limit, not an open-ended spin
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum().item()) == 56.0  # the context is still usable
