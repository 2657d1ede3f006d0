"""GPU parity of the whole FP8 MoE layer at the benchmark geometry
(H=2048, E=128, I=768, top-8) against the oracle: routing indices bit-exact,
outputs within max-abs 2e-2 and relative-L2 1e-2."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import assert_close, experts_to_oracle, from_bf16, to_bf16, ulps_bf16  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

E, I, H, K = 128, 768, 2048, 8


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth
    lw = synth.make_layer(E, I, H, seed=1, device="cuda")
    return lw, experts_to_oracle(lw.experts), experts_to_oracle(lw.shared)


def _x(T, seed):
    rng = np.random.default_rng(seed)
    return O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))


@pytest.mark.parametrize("T", [1, 8, 16, 32, 64])
def test_layer_matches_oracle(layer, T):
    from d3moe import ops
    lw, ex, sh = layer
    x = _x(T, T)
    out, ids, w = ops.moe_layer(to_bf16(x), lw.router, lw.experts, lw.shared, K, return_routing=True)
    ref, ids_o, w_o = O.moe_layer(x, from_bf16(lw.router), ex, sh, K)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    assert ulps_bf16(from_bf16(w), w_o).max() <= 1
    assert_close(from_bf16(out), ref, what=f"moe_layer T={T}")


@pytest.mark.parametrize("T", [64, 130])
def test_hot_expert_bias(layer, T):
    """A router bias that sends every token to the same few experts: one
    expert sees all T tokens (full 64-token groups, and a second group when
    T > 64)."""
    from d3moe import ops
    lw, ex, sh = layer
    bias = np.zeros(E, np.float32)
    bias[[5, 77, 3]] = 30.0
    x = _x(T, 100 + T)
    bt = torch.from_numpy(bias).cuda()
    out, ids, w = ops.moe_layer(to_bf16(x), lw.router, lw.experts, lw.shared, K, router_bias=bt,
                                return_routing=True)
    ref, ids_o, w_o = O.moe_layer(x, from_bf16(lw.router), ex, sh, K, bias=bias)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    assert_close(from_bf16(out), ref, what=f"hot experts T={T}")


def test_experts_api_parts_match_layer(layer):
    """moe_parts-style routed/shared outputs recombine to the fused layer."""
    from d3moe import ops
    from d3moe.model import MoE
    lw, _, _ = layer

    class L:
        experts = lw.experts
        shared_expert = lw.shared
        router_weight = lw.router

    x = to_bf16(_x(16, 3))
    m = MoE()
    routed, shared, gate = m.moe_parts(x, L)
    fused = m.moe(x, L)
    np.testing.assert_array_equal(from_bf16(ops.combine_experts(routed, shared, gate)), from_bf16(fused))


def test_cuda_graph_replay_matches_eager(layer):
    from d3moe import ops
    lw, _, _ = layer
    T = 64
    ws = ops.moe_workspace(T, K, E, I, H, True, "cuda")
    static_x = to_bf16(_x(T, 7))
    out = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.moe_layer(static_x, lw.router, lw.experts, lw.shared, K, workspace=ws, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.moe_layer(static_x, lw.router, lw.experts, lw.shared, K, workspace=ws, out=out)
    for seed in (11, 12, 13):
        xn = to_bf16(_x(T, seed))
        static_x.copy_(xn)
        g.replay()
        torch.cuda.synchronize()
        eager = ops.moe_layer(xn, lw.router, lw.experts, lw.shared, K)
        np.testing.assert_array_equal(from_bf16(out), from_bf16(eager))


def test_status_word_stays_ok(layer):
    from d3moe import ops
    lw, _, _ = layer
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.moe_layer(to_bf16(_x(32, 9)), lw.router, lw.experts, lw.shared, K, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
