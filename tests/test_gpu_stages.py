"""GPU parity of the stage-level entry points d3_moe_gate_up_silu and
d3_moe_down_combine (the reference's expert_up_kernel / down split,
src/drama3/kernels.py:290-322, 344): the pair, with other work queued between
the two calls, gives moe_experts' routed and shared outputs bit for bit, on
the decode engine and on the tcgen05 prefill path."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

E, I, H, K = 128, 768, 2048, 8


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth
    return synth.make_layer(E, I, H, seed=57, device="cuda")


def routing(T, seed):
    from d3moe import ops
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g, device="cuda")
    w, ids = ops.route_topk(logits, K, weights_dtype=torch.bfloat16)
    return x, ids, w


@pytest.mark.parametrize("T,prefill,with_shared", [(1, False, True), (64, False, True), (64, False, False),
                                                   (2048, True, True), (700, True, False)])
def test_stage_pair_equals_moe_experts(layer, T, prefill, with_shared):
    from d3moe import ops
    x, ids, w = routing(T, seed=T + 3)
    sh = layer.shared if with_shared else None
    with ops.prefill_min_tokens(1 if prefill else 1 << 30):
        ref_routed, ref_shared = ops.moe_experts(x, ids, w, layer.experts, sh)
        ws = ops.moe_gate_up_silu(x, ids, layer.experts, sh)
        filler = torch.randn((1024, 1024), device="cuda") @ torch.randn((1024, 1024), device="cuda")
        routed, shared_out = ops.moe_down_combine(w, ws, layer.experts, sh)
    torch.cuda.synchronize()
    assert filler.isfinite().all()
    assert torch.equal(routed, ref_routed)
    if with_shared:
        assert torch.equal(shared_out, ref_shared)
    else:
        assert shared_out is None


def test_stage_checks(layer):
    from d3moe import ops
    from d3moe._lib import D3Error
    x, ids, w = routing(16, seed=1)
    ws = ops.moe_gate_up_silu(x, ids, layer.experts, layer.shared)
    with pytest.raises(D3Error):
        ops.moe_down_combine(w, ws[:16], layer.experts, layer.shared)  # workspace too small
