"""The workspace-free weight-only FP8 GEMV (d3_fp8_gemv_noalloc).

Some callers cannot hand this library a workspace: a host runtime that gives
a plugin only its inputs, outputs and a stream, and does not let it allocate
device memory while a request runs. For them the library keeps the GEMV's
scratch in a fixed array of its own. These tests call that entry point through
the C ABI and check it against the workspace entry point (d3_fp8_gemv) on
calls in a row with different shapes, in both orders (a small call before a
large one and after it, and an N whose last 128-row tile is partial), so each
later call proves that whatever the earlier calls left in the shared array
does not leak into its result. The array's status word, read through
d3_fp8_gemv_noalloc_status, must report no timeout and read back cleared.
This file is collected last on purpose.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import assert_close, from_bf16, to_bf16, to_fp8  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402


def _case(T, N, K, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    q, s = O.quantize_weight_blocks(w)
    x = O.bf16_round(rng.standard_normal((T, K)).astype(np.float32))
    return x, q, s


def _within_rounding_bound(got, x, q, s, N, what):
    """The float64 value of the same dequantise-then-matmul, correctly rounded
    to bf16 up to fp32 summation-order noise (half a bf16 ulp + 2^-16 of the
    output rms): the bound every dense GEMV test of this library uses."""
    exact = x.astype(np.float64) @ O.dequant_blocks(q, s)[:N].astype(np.float64).T
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 1e-30))) - 7)
    bound = 0.5 * ulp + np.sqrt((exact ** 2).mean()) * 2.0 ** -16
    excess = np.abs(got - exact) - bound
    assert (excess <= 0).all(), f"{what}: {float(excess.max())} above the rounding bound"


def _noalloc(x, wq, s, N):
    from d3moe import _lib, ops
    T, K = x.shape
    y = torch.empty((T, N), dtype=torch.bfloat16, device=x.device)
    _lib.call("d3_fp8_gemv_noalloc", x.data_ptr(), x.stride(0), wq.data_ptr(), s.data_ptr(), T, N, K,
              y.data_ptr(), y.stride(0), ops._stream(x.device))
    return y


def _noalloc_status(device):
    from d3moe import _lib, ops
    st = torch.full((1,), -1, dtype=torch.int32, device=device)
    _lib.call("d3_fp8_gemv_noalloc_status", st.data_ptr(), ops._stream(device))
    torch.cuda.synchronize()
    return int(st.item())


def test_noalloc_gemv_matches_workspace_gemv_on_consecutive_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import ops
    cases = ((64, 4096, 2048, 1), (13, 2048, 4096, 2), (1, 4096 - 64, 4096, 3),
             (1, 2048, 2048, 4), (64, 4096, 4096, 5))
    for T, N, K, seed in cases:
        xn, qn, sn = _case(T, N, K, seed)
        x, wq, s = to_bf16(xn), to_fp8(qn), torch.from_numpy(sn).cuda()
        got = from_bf16(_noalloc(x, wq, s, N))
        ref = from_bf16(ops.fp8_gemv(x, wq, s, n=N))
        torch.cuda.synchronize()
        # the two entry points add the same products in different orders, so
        # each is held to the exact value's rounding bound, and to each other
        # within the layer tolerance
        what = f"noalloc gemv T={T} N={N} K={K}"
        _within_rounding_bound(got, xn, qn, sn, N, what)
        _within_rounding_bound(ref, xn, qn, sn, N, what + " (workspace entry point)")
        assert_close(got, ref, what=what)
    dev = torch.device("cuda")
    assert _noalloc_status(dev) == 0, "a bounded wait of the no-allocation GEMV timed out"
    assert _noalloc_status(dev) == 0, "the status word was not cleared by the read"


def test_noalloc_gemv_rejects_sizes_beyond_its_scratch():
    from d3moe import _lib
    with pytest.raises(ValueError, match="fixed scratch limits"):
        _lib.call("d3_fp8_gemv_noalloc", 16, 2048, 16, 16, 65, 4096, 2048, 16, 4096, None)
    with pytest.raises(ValueError, match="fixed scratch limits"):
        _lib.call("d3_fp8_gemv_noalloc", 16, 8192, 16, 16, 8, 4096, 8192, 16, 4096, None)
