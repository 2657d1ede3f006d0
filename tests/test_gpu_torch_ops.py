"""GPU check of the torch.library registrations: each operator gives the
d3moe.ops function's result bit for bit, and torch.library.opcheck accepts its
fake implementation (and, where no input is FP8, its schema) against the
real kernel. opcheck's schema check runs arithmetic on the inputs, which
torch does not implement for float8_e4m3fn tensors."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

E, I, H, K = 128, 768, 2048, 8


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth, torch_ops  # noqa: F401
    return synth.make_layer(E, I, H, seed=61, device="cuda")


def _expert_tensors(ex):
    return ex.w13_weight, ex.w13_scale_inv, ex.w2_weight, ex.w2_scale_inv


def test_ops_match_and_pass_opcheck(layer):
    from d3moe import ops
    T = 64
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g, device="cuda")
    w, ids = torch.ops.d3moe.route_topk(logits, K)
    w_ref, ids_ref = ops.route_topk(logits, K, weights_dtype=torch.bfloat16)
    assert torch.equal(w, w_ref) and torch.equal(ids, ids_ref)
    ex = _expert_tensors(layer.experts)
    y = torch.ops.d3moe.moe_experts(x, ids, w, *ex, 0)
    y_ref, _ = ops.moe_experts(x, ids, w, layer.experts)
    assert torch.equal(y, y_ref)
    sh = _expert_tensors(layer.shared)
    out = torch.ops.d3moe.moe_layer(x, layer.router, *ex, *sh, K, 0)
    assert torch.equal(out, ops.moe_layer(x, layer.router, layer.experts, layer.shared, K))
    q, s = torch.ops.d3moe.quant_act_fp8(x, True)
    q_ref, s_ref = ops.quant_act_fp8(x, transposed=True)
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8)) and torch.equal(s, s_ref)
    torch.library.opcheck(torch.ops.d3moe.route_topk.default, (logits, K),
                          test_utils=("test_schema", "test_faketensor"))
    fake = ("test_faketensor",)
    torch.library.opcheck(torch.ops.d3moe.moe_experts.default, (x, ids, w, *ex, 0), test_utils=fake)
    torch.library.opcheck(torch.ops.d3moe.quant_act_fp8.default, (x, False), test_utils=fake)


def test_fp8_gemv_and_exit(layer):
    from d3moe import ops
    T, N = 8, 4096
    x = torch.randn((T, H), device="cuda").to(torch.bfloat16)
    wq, s = ops.fp8_quantize_weight(torch.randn((N, H), device="cuda").to(torch.bfloat16) * 0.02)
    assert torch.equal(torch.ops.d3moe.fp8_gemv(x, wq, s), ops.fp8_gemv(x, wq, s))
    torch.library.opcheck(torch.ops.d3moe.fp8_gemv.default, (x, wq, s), test_utils=("test_faketensor",))
    routed, shared = x.clone(), torch.randn_like(x)
    gate = torch.randn((T, 1), device="cuda").to(torch.bfloat16)
    res_a = torch.randn_like(x)
    res_b = res_a.clone()
    nw = torch.randn((H,), device="cuda").to(torch.bfloat16) * 0.1
    a = torch.ops.d3moe.combine_experts_add_norm(routed, shared, gate, res_a, nw, 1e-6)
    b = ops.combine_experts_add_norm(routed, shared, gate, res_b, nw, 1e-6)
    assert torch.equal(a, b) and torch.equal(res_a, res_b)
