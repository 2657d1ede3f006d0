"""GPU checks of the model-level drop-in (d3moe.model.MoE, d3moe.kernels.linear)
driven the way the reference drives it: a layer object with the reference's
own attribute names (src/drama3/model.py:195-245, 495-517) -- experts,
gate.weight, shared_expert_gate.weight and a bf16 shared expert with
gate_proj / up_proj / down_proj -- is converted once on first use and gives
the oracle's layer output; moe() equals moe_parts() + combine_experts(), and
`decode` changes nothing."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import assert_close, experts_to_oracle, from_bf16, to_bf16  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

E, I, H, K = 128, 768, 2048, 8


def _lin(w):
    return SimpleNamespace(weight=w)


@pytest.fixture(scope="module")
def ref_layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth
    g = torch.Generator(device="cpu").manual_seed(21)
    experts = synth.make_experts(E, I, H, seed=21, device="cuda")
    rnd = lambda *shape: (torch.randn(shape, generator=g) * 0.02).to(torch.bfloat16).cuda()  # noqa: E731
    shared = SimpleNamespace(gate_proj=_lin(rnd(I, H)), up_proj=_lin(rnd(I, H)), down_proj=_lin(rnd(H, I)))
    return SimpleNamespace(experts=experts, gate=_lin(rnd(E, H)), shared_expert_gate=_lin(rnd(1, H)),
                           shared_expert=shared)


@pytest.mark.parametrize("T", [8, 64])
def test_reference_layer_object_matches_oracle(ref_layer, T):
    from d3moe import model, ops
    m = model.MoE()
    rng = np.random.default_rng(T)
    x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    out = m.moe(to_bf16(x), ref_layer, decode=True)
    view = ref_layer._d3moe_view  # the one-time conversion, cached on the layer
    assert view.router_weight.shape == (E + 1, H)
    assert torch.equal(view.router_weight[:E], ref_layer.gate.weight)
    assert torch.equal(view.router_weight[E], ref_layer.shared_expert_gate.weight[0])
    ref, _, _ = O.moe_layer(x, from_bf16(view.router_weight), experts_to_oracle(ref_layer.experts),
                            experts_to_oracle(view.shared_expert), K)
    assert_close(from_bf16(out), ref, what=f"reference layer object T={T}")
    # decode selects no other computation; moe() == moe_parts() + combine
    assert torch.equal(m.moe(to_bf16(x), ref_layer, decode=False), out)
    routed, shared, gate = m.moe_parts(to_bf16(x), ref_layer)
    assert torch.equal(ops.combine_experts(routed, shared, gate), out)
    # the shared expert is the bf16 one quantised per 128x128 block
    w13 = torch.cat((ref_layer.shared_expert.gate_proj.weight, ref_layer.shared_expert.up_proj.weight))
    deq = (view.shared_expert.w13_weight[0].float().view(2 * I // 128, 128, H // 128, 128)
           * view.shared_expert.w13_scale_inv[0][:, None, :, None]).reshape(2 * I, H)
    assert (deq - w13.float()).abs().max() <= w13.float().abs().max() / 16


def test_biased_router_moe_parts_match_moe(ref_layer):
    """With a per-expert router bias (N(0,1), as in the 24-layer benchmark
    stack) moe_parts routes on the same biased bf16 logits as moe(), so
    moe_parts + combine_experts equals moe() bit for bit."""
    from d3moe import model, ops
    view = model.layer_view(ref_layer)
    bias = torch.randn(E, generator=torch.Generator(device="cpu").manual_seed(5)).cuda()
    layer = SimpleNamespace(experts=view.experts, shared_expert=view.shared_expert,
                            router_weight=view.router_weight, router_bias=bias)
    m = model.MoE()
    x = torch.randn((64, H), generator=torch.Generator(device="cpu").manual_seed(6)).to(torch.bfloat16).cuda()
    out = m.moe(x, layer)
    routed, shared, gate = m.moe_parts(x, layer)
    assert torch.equal(ops.combine_experts(routed, shared, gate), out)


def test_linear_is_the_fp8_projection(ref_layer):
    """kernels.linear(x, weight) (kernels.py:274-287): the weight is quantised
    once on first use and every call is the FP8 GEMV of that registration."""
    from d3moe import experimental_fp8, kernels
    w = ref_layer.gate.weight
    x = torch.randn((16, H), generator=torch.Generator(device="cpu").manual_seed(3)).to(torch.bfloat16).cuda()
    y = kernels.linear(x, w)
    assert w.data_ptr() in experimental_fp8.WEIGHTS
    _, q, s = experimental_fp8.WEIGHTS[w.data_ptr()][:3]
    ref = O.fp8_gemv(from_bf16(x), q.view(torch.uint8).cpu().numpy(), s.cpu().numpy(), n=E)
    assert_close(from_bf16(y), ref, what="linear")
    assert torch.equal(kernels.linear(x, w), y)
