"""The path's operators registered with torch.library (namespace "d3moe").

Registered operators carry a schema and a fake (meta) implementation, so a
model that calls them can be traced (FakeTensor / meta tensors, torch.fx,
torch.export) and stays one opaque node per call. The reference registers its
own CUDA operators this way (src/drama3/ops/slot_attention.py:350-460). Each
operator runs the same C-ABI entry point as the function of the same name in
d3moe.ops; there is no CPU implementation.

Expert weights enter as tensors (w13, s13, w2, s2) with gate_up_order 0 for
w13 rows [gate | up] (the checkpoint order) and 1 for [up | gate]
(FlashInfer's order, src/drama3/model.py:196-201).
"""

from __future__ import annotations

import torch

from . import ops

FP8 = torch.float8_e4m3fn
_ORDERS = ("gate_up", "up_gate")


def _view(w13, s13, w2, s2, gate_up_order: int) -> ops.ExpertView:
    if gate_up_order not in (0, 1):
        raise ValueError("gate_up_order must be 0 (gate_up) or 1 (up_gate)")
    return ops.ExpertView(tensors=(w13, s13, w2, s2), gate_up_order=_ORDERS[gate_up_order])


@torch.library.custom_op("d3moe::quant_act_fp8", mutates_args=())
def quant_act_fp8(x: torch.Tensor, transposed: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """prepare_moe_input's activation quantiser (src/drama3/moe_input.py:24-27)."""
    return ops.quant_act_fp8(x, transposed=transposed)


@quant_act_fp8.register_fake
def _(x, transposed):
    T, H = x.shape
    s = (H // 128, T) if transposed else (T, H // 128)
    return x.new_empty((T, H), dtype=FP8), x.new_empty(s, dtype=torch.float32)


@torch.library.custom_op("d3moe::route_topk", mutates_args=())
def route_topk(logits: torch.Tensor, k: int, bias: torch.Tensor | None = None
               ) -> tuple[torch.Tensor, torch.Tensor]:
    """route (src/drama3/kernels.py:360-383): (weights bf16 [T,k], ids int64 [T,k])."""
    return ops.route_topk(logits, k, bias=bias, weights_dtype=torch.bfloat16)


@route_topk.register_fake
def _(logits, k, bias=None):
    T = logits.shape[0]
    return (logits.new_empty((T, k), dtype=torch.bfloat16),
            logits.new_empty((T, k), dtype=torch.int64))


@torch.library.custom_op("d3moe::moe_experts", mutates_args=())
def moe_experts(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
                gate_up_order: int = 0) -> torch.Tensor:
    """Routed expert output bf16 [T,H] (small_batch_moe / native_moe,
    src/drama3/kernels.py:325-357, 702-779)."""
    routed, _ = ops.moe_experts(x, topk_ids, topk_weights, _view(w13, s13, w2, s2, gate_up_order))
    return routed


@moe_experts.register_fake
def _(x, topk_ids, topk_weights, w13, s13, w2, s2, gate_up_order=0):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


@torch.library.custom_op("d3moe::moe_layer", mutates_args=())
def moe_layer(x: torch.Tensor, router_weight: torch.Tensor,
              w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
              sh_w13: torch.Tensor, sh_s13: torch.Tensor, sh_w2: torch.Tensor, sh_s2: torch.Tensor,
              k: int = 8, gate_up_order: int = 0) -> torch.Tensor:
    """Whole MoE layer (DramaModel.moe, src/drama3/model.py:485-541): router
    rows [E + 1, H] (the last row is the shared-expert gate), routed and shared
    experts, out = routed + bf16(shared * bf16(sigmoid(gate)))."""
    return ops.moe_layer(x, router_weight, _view(w13, s13, w2, s2, gate_up_order),
                         _view(sh_w13, sh_s13, sh_w2, sh_s2, gate_up_order), k)


@moe_layer.register_fake
def _(x, router_weight, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, k=8, gate_up_order=0):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


@torch.library.custom_op("d3moe::fp8_gemv", mutates_args=())
def fp8_gemv(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Weight-only FP8 projection y bf16 [T,N] (experimental_fp8.linear,
    src/drama3/experimental_fp8.py:56-79)."""
    return ops.fp8_gemv(x, wq, scales)


@fp8_gemv.register_fake
def _(x, wq, scales):
    return x.new_empty((x.shape[0], wq.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("d3moe::combine_experts_add_norm", mutates_args=("residual",))
def combine_experts_add_norm(routed: torch.Tensor, shared: torch.Tensor, gate: torch.Tensor,
                             residual: torch.Tensor, weight: torch.Tensor, epsilon: float
                             ) -> torch.Tensor:
    """Layer exit (src/drama3/kernels.py:448-499): residual is updated in
    place and RMSNorm(residual) * (1 + weight) is returned."""
    return ops.combine_experts_add_norm(routed, shared, gate, residual, weight, epsilon)


@combine_experts_add_norm.register_fake
def _(routed, shared, gate, residual, weight, epsilon):
    return residual.new_empty(residual.shape, dtype=torch.bfloat16)
