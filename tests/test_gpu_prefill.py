"""GPU parity of the prefill path: both expert GEMMs on the tcgen05 grouped
kernel (128-token x 256-column tiles, FP8 E4M3 MMAs into TMEM, per-128-K-block
fp32 scale promotion). The path is forced with a low token threshold so the
oracle can check it at sizes it finishes in seconds; at the benchmark's 8192
tokens it is checked against the decode engine (an independent kernel over the
same workspace layout): routing identical, values within the parity tolerance,
outputs bit-identical across repeated calls."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import assert_close, device_logits_routing, experts_to_oracle, from_bf16, to_bf16  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

E, I, H, K = 128, 768, 2048, 8


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth
    lw = synth.make_layer(E, I, H, seed=11, device="cuda")
    return lw, experts_to_oracle(lw.experts), experts_to_oracle(lw.shared)


def _x(T, seed, h=H):
    rng = np.random.default_rng(seed)
    return O.bf16_round(rng.standard_normal((T, h)).astype(np.float32))


@pytest.mark.parametrize("T", [200, 256])
def test_prefill_layer_matches_oracle(layer, T):
    from d3moe import ops
    lw, ex, sh = layer
    x = _x(T, 1000 + T)
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    with ops.prefill_min_tokens(1):
        out, ids, w = ops.moe_layer(to_bf16(x), lw.router, lw.experts, lw.shared, K,
                                    return_routing=True, status=status)
    lg, ids_o, w_o = device_logits_routing(x, lw.router, E, K)
    routed, shared = O.moe_experts(x, ids_o, w_o, ex, sh, rows_bf16=True)
    ref = O.combine_experts(routed, shared, lg[:, E])
    assert int(status[0]) == 0
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    assert_close(from_bf16(out), ref, what=f"prefill layer T={T}")


def test_prefill_hot_experts_span_tiles(layer):
    """Three experts take every token: each expert's rows span several
    128-row tiles with a ragged last tile, and the other experts are empty."""
    from d3moe import ops
    lw, ex, sh = layer
    T = 300
    bias = np.zeros(E, np.float32)
    bias[[9, 64, 127]] = 30.0
    x = _x(T, 7)
    with ops.prefill_min_tokens(1):
        out, ids, _ = ops.moe_layer(to_bf16(x), lw.router, lw.experts, lw.shared, K,
                                    router_bias=torch.from_numpy(bias).cuda(), return_routing=True)
    lg, ids_o, w_o = device_logits_routing(x, lw.router, E, K, bias=bias)
    routed, shared = O.moe_experts(x, ids_o, w_o, ex, sh, rows_bf16=True)
    ref = O.combine_experts(routed, shared, lg[:, E])
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    assert_close(from_bf16(out), ref, what="prefill hot experts")


def test_prefill_experts_other_geometry():
    """moe_experts at E=8, I=256, H=512, top-2 with given routing (and no
    shared expert): two n tiles per GEMM, experts of 0..T tokens."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import ops, synth
    e_, i_, h_, k_, T = 8, 256, 512, 2, 333
    ew = synth.make_experts(e_, i_, h_, seed=3, device="cuda")
    exo = experts_to_oracle(ew)
    rng = np.random.default_rng(5)
    ids = np.stack([rng.choice([0, 2, 3, 7], size=2, replace=False) for _ in range(T)]).astype(np.int64)
    w = O.bf16_round(rng.uniform(0.1, 1.0, (T, k_)).astype(np.float32))
    x = _x(T, 6, h_)
    with ops.prefill_min_tokens(1):
        routed, shared = ops.moe_experts(to_bf16(x), torch.from_numpy(ids).cuda(), to_bf16(w), ew)
    assert shared is None
    ref, _ = O.moe_experts(x, ids, w, exo, rows_bf16=True)
    assert_close(from_bf16(routed), ref, what="prefill experts E=8")


@pytest.mark.parametrize("T", [2048, 8192])
def test_prefill_matches_decode_engine_at_scale(layer, T):
    """At prefill sizes the oracle is too slow; the decode engine (checked
    against the oracle by the decode tests) is the cross-check. Routing is
    computed once, so both paths see the same pairs."""
    from d3moe import ops
    lw, _, _ = layer
    g = torch.Generator(device="cuda")
    g.manual_seed(T)
    x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    with ops.prefill_min_tokens(1 << 30):
        ref, ids_e, _ = ops.moe_layer(x, lw.router, lw.experts, lw.shared, K, return_routing=True)
    with ops.prefill_min_tokens(1):
        out, ids_t, _ = ops.moe_layer(x, lw.router, lw.experts, lw.shared, K, return_routing=True)
        out2 = ops.moe_layer(x, lw.router, lw.experts, lw.shared, K)
    torch.testing.assert_close(ids_t, ids_e, rtol=0, atol=0)
    assert torch.equal(out, out2), "prefill path is not deterministic"
    assert_close(from_bf16(out), from_bf16(ref), what=f"prefill vs engine T={T}")


def test_prefill_graph_replay(layer):
    """The prefill path is capturable: a graph replay reproduces the eager
    output bit for bit."""
    from d3moe import ops
    lw, _, _ = layer
    T = 1536
    x = torch.randn((T, H), device="cuda").to(torch.bfloat16)
    ws = ops.moe_workspace(T, K, E, I, H, True, "cuda")
    out = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    with ops.prefill_min_tokens(1):
        eager = ops.moe_layer(x, lw.router, lw.experts, lw.shared, K, workspace=ws).clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ops.moe_layer(x, lw.router, lw.experts, lw.shared, K, workspace=ws, out=out)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ops.moe_layer(x, lw.router, lw.experts, lw.shared, K, workspace=ws, out=out)
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
    assert torch.equal(out, eager)
