"""The torch.library registrations (d3moe.torch_ops) on meta tensors: schemas,
fake implementations (output shapes and dtypes) and tracing into one graph
node per call. No kernel runs here."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from d3moe import torch_ops  # noqa: E402,F401  (registers the operators)

FP8 = torch.float8_e4m3fn
T, H, E, I, K = 16, 2048, 128, 768, 8


def meta(shape, dtype=torch.float32):
    return torch.empty(shape, dtype=dtype, device="meta")


def experts():
    return (meta((E, 2 * I, H), FP8), meta((E, 2 * I // 128, H // 128)),
            meta((E, H, I), FP8), meta((E, H // 128, I // 128)))


def test_fake_shapes():
    x = meta((T, H), torch.bfloat16)
    q, s = torch.ops.d3moe.quant_act_fp8(x, True)
    assert (q.shape, q.dtype, s.shape, s.dtype) == ((T, H), FP8, (H // 128, T), torch.float32)
    q, s = torch.ops.d3moe.quant_act_fp8(x, False)
    assert s.shape == (T, H // 128)
    w, ids = torch.ops.d3moe.route_topk(meta((T, E)), K)
    assert (w.shape, w.dtype, ids.dtype) == ((T, K), torch.bfloat16, torch.int64)
    y = torch.ops.d3moe.moe_experts(x, ids, w, *experts(), 0)
    assert (y.shape, y.dtype) == ((T, H), torch.bfloat16)
    sh = (meta((1, 2 * I, H), FP8), meta((1, 2 * I // 128, H // 128)), meta((1, H, I), FP8),
          meta((1, H // 128, I // 128)))
    y = torch.ops.d3moe.moe_layer(x, meta((E + 1, H), torch.bfloat16), *experts(), *sh, K, 1)
    assert y.shape == (T, H)
    y = torch.ops.d3moe.fp8_gemv(x, meta((4096, H), FP8), meta((32, 16)))
    assert (y.shape, y.dtype) == ((T, 4096), torch.bfloat16)
    y = torch.ops.d3moe.combine_experts_add_norm(x, x, meta((T, 1), torch.bfloat16),
                                                 meta((T, H), torch.bfloat16), meta((H,), torch.bfloat16), 1e-6)
    assert y.shape == (T, H)


def test_schemas():
    s = str(torch.ops.d3moe.combine_experts_add_norm.default._schema)
    assert "Tensor(a3!) residual" in s  # the residual is declared as mutated
    for name in ("quant_act_fp8", "route_topk", "moe_experts", "moe_layer", "fp8_gemv"):
        assert "!" not in str(getattr(torch.ops.d3moe, name).default._schema), name


def test_traces_to_one_node_per_call():
    from torch.fx.experimental.proxy_tensor import make_fx

    def layer(x, logits, w13, s13, w2, s2):
        w, ids = torch.ops.d3moe.route_topk(logits, K)
        return torch.ops.d3moe.moe_experts(x, ids, w, w13, s13, w2, s2, 0)

    g = make_fx(layer, tracing_mode="fake")(meta((T, H), torch.bfloat16), meta((T, E)), *experts())
    targets = [n.target for n in g.graph.nodes if n.op == "call_function"]
    assert torch.ops.d3moe.route_topk.default in targets
    assert torch.ops.d3moe.moe_experts.default in targets
