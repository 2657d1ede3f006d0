"""GPU parity of the gated FP8 projection (the reference's gated_gemv,
src/drama3/fused_projection.py:9-60, on block-quantised FP8 weights) at the
real Drama-3 out-projection shape (2048 x 4096) and the benchmark shapes."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import assert_close, from_bf16, to_bf16, to_fp8  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402


@pytest.fixture(scope="module")
def d3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import experimental_fp8, fused_projection, ops
    return ops, fused_projection, experimental_fp8


@pytest.mark.parametrize("mode", ["swiglu", "sigmoid"])
@pytest.mark.parametrize("T,N,K", [(1, 2048, 4096), (1, 4096, 2048), (8, 2048, 4096), (64, 2048, 2048)])
def test_gated_gemv_matches_oracle(d3, mode, T, N, K):
    ops = d3[0]
    rng = np.random.default_rng(N + K + T)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    q, s = O.quantize_weight_blocks(w)
    x = O.bf16_round(rng.standard_normal((T, K)).astype(np.float32))
    g = O.bf16_round((rng.standard_normal((T, K)) * 2.0).astype(np.float32))
    y = ops.fp8_gated_gemv(to_bf16(x), to_bf16(g), to_fp8(q), torch.from_numpy(s).cuda(), mode)
    ref = O.fp8_gemv(O.gated_input(x, g, mode), q, s)
    assert_close(from_bf16(y), ref, what=f"gated gemv {mode}")


def test_gated_gemv_drop_in(d3):
    ops, fp, reg = d3
    rng = np.random.default_rng(3)
    N, K = 2048, 4096
    w = to_bf16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    reg.register(w)
    _, q, s = reg.WEIGHTS[w.data_ptr()][:3]
    x = to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    g = to_bf16(rng.standard_normal(K).astype(np.float32))
    for mode in ("swiglu", "sigmoid"):
        a = fp.gated_gemv(x, g, w, mode)
        b = ops.fp8_gated_gemv(x, g.reshape(1, -1), q, s, mode)
        torch.cuda.synchronize()
        assert a.shape == (1, N) and torch.equal(a, b)
    with pytest.raises(ValueError):
        fp.gated_gemv(torch.cat([x, x]), g, w, "swiglu")
    with pytest.raises(ValueError):
        fp.gated_gemv(x, g, w, "gelu")
