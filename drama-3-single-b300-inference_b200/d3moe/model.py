"""Model-level MoE entry points with the reference's signatures
(DramaModel.moe / moe_parts / routed_moe, src/drama3/model.py:485-583).

`layer` is either the reference's own MoE layer object or this package's
container:
  reference layer (src/drama3/model.py:195-245, 495-517):
    experts                               routed FP8 experts (w13_weight,
                                          w13_scale_inv, w2_weight, w2_scale_inv)
    gate.weight                           bf16 [E, H] router
    shared_expert_gate.weight             bf16 [1, H] shared-expert gate
    shared_expert.gate_proj / up_proj / down_proj .weight
                                          bf16 shared expert (or its
                                          packed_gate_up [2I, H])
  This package's container:
    experts, shared_expert (FP8, E = 1), router_weight bf16 [E+1, H],
    router_bias (optional) f32 [E], added to the router logits.
A reference layer is converted once, on first use, and the result is cached
on the layer (`_d3moe_view`): the router and shared-gate rows are packed into
[E+1, H] (the packed projection of model.py:236-245) and the bf16 shared
expert is quantised into 128x128 block-scaled FP8, the format the benchmark
configurations give the shared expert.

Routing always runs on the device (route_topk); the routed and shared experts
run in the same launches of the expert engine. No host synchronisation, so a
decode step built from these calls is CUDA-graph capturable.

`decode` is accepted as in the reference. There it chooses the routing code
(the Triton route kernel or torch softmax/top-k, model.py:522-528) and
whether the shared expert runs on a side stream (model.py:506-517). Here both
routings are the same computation (fp32 softmax over the bf16 logits, top-k
with ties to the lower id, renormalised) and the shared expert already runs
inside the routed experts' launches, so `decode` changes no result and no
kernel: the kernel choice follows the token count, as the reference's own
small_moe_max_batch / tuned-prefill switch does.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch

from . import ops
from .synth import ExpertWeights


def _weight(module_or_tensor) -> torch.Tensor:
    return module_or_tensor.weight if hasattr(module_or_tensor, "weight") else module_or_tensor


def _quantize_expert(gate_up: torch.Tensor, down: torch.Tensor) -> ExpertWeights:
    """bf16 gate_up [2I, H] (rows [gate | up]) and down [H, I] -> one FP8
    expert with 128x128 block scales (experimental_fp8.py:10-18 quantiser)."""
    w13, s13 = ops.fp8_quantize_weight(gate_up.to(torch.bfloat16).contiguous())
    w2, s2 = ops.fp8_quantize_weight(down.to(torch.bfloat16).contiguous())
    return ExpertWeights(w13[None], s13[None], w2[None], s2[None])


def layer_view(layer):
    """The (experts, shared_expert, router_weight, router_bias) view of `layer`
    that the kernels take; reference layers are converted once and cached."""
    if hasattr(layer, "router_weight"):
        return layer
    view = getattr(layer, "_d3moe_view", None)
    if view is not None:
        return view
    router = _weight(layer.gate)
    gate = _weight(layer.shared_expert_gate)
    router_weight = torch.cat((router, gate.reshape(1, -1)), 0).to(torch.bfloat16).contiguous()
    sh = layer.shared_expert
    packed = getattr(sh, "packed_gate_up", None)
    if packed is None:
        packed = torch.cat((_weight(sh.gate_proj), _weight(sh.up_proj)), 0)
    shared = _quantize_expert(packed, _weight(sh.down_proj))
    view = SimpleNamespace(experts=layer.experts, shared_expert=shared, router_weight=router_weight,
                           router_bias=getattr(layer, "router_bias", None))
    layer._d3moe_view = view
    return view


class MoE:
    """Holds per-layer workspaces so repeated calls (and graph replays) reuse
    the same device buffers."""

    def __init__(self, top_k: int = 8, padding_start: int | None = None):
        """padding_start: the reserved-slot boundary of the padding-router rule
        (the reference sets it to slots // 2 when reserved_padding_router is on,
        src/drama3/model.py:546-553); None ignores row_slots like the reference
        does with the rule off."""
        self.top_k = top_k
        self.padding_start = padding_start
        self._ws: dict = {}

    def _workspace(self, T: int, layer) -> torch.Tensor:
        ex = layer.experts
        E, I2, H = ex.w13_weight.shape
        key = (T, E, I2, H, ex.w13_weight.device)
        ws = self._ws.get(key)
        if ws is None:
            ws = ops.moe_workspace(T, self.top_k, E, I2 // 2, H, True, ex.w13_weight.device)
            self._ws[key] = ws
        return ws

    def _padding(self, row_slots):
        if row_slots is None or self.padding_start is None:
            return None, None
        return row_slots, self.padding_start

    def moe(self, x: torch.Tensor, layer, decode: bool = False, *, row_slots=None) -> torch.Tensor:
        """out = routed + bf16(shared * bf16(sigmoid(gate))) in one pipeline."""
        layer = layer_view(layer)
        slots, start = self._padding(row_slots)
        return ops.moe_layer(x, layer.router_weight, layer.experts, layer.shared_expert, self.top_k,
                             router_bias=getattr(layer, "router_bias", None),
                             workspace=self._workspace(len(x), layer), row_slots=slots,
                             padding_start=start)

    def moe_add_norm(self, x: torch.Tensor, layer, residual: torch.Tensor, norm_weight: torch.Tensor,
                     eps: float = 1e-6, *, keep=None, inverse=None, row_slots=None) -> torch.Tensor:
        """The mixed decode + packed-prefill layer step in one call
        (src/drama3/mixed_model.py:200-246): moe_parts over x[keep] with the
        padding-router rule on row_slots, then combine_experts_add_norm(_inverse)
        into residual. Returns the normalised rows [len(residual), H]."""
        layer = layer_view(layer)
        slots, start = self._padding(row_slots)
        T = len(keep) if keep is not None else len(x)
        return ops.moe_layer(x, layer.router_weight, layer.experts, layer.shared_expert, self.top_k,
                             router_bias=getattr(layer, "router_bias", None),
                             workspace=self._workspace(T, layer), residual=residual,
                             norm_weight=norm_weight, norm_eps=eps, keep=keep, inverse=inverse,
                             row_slots=slots, padding_start=start)

    def moe_parts(self, x: torch.Tensor, layer, decode: bool = False, *, row_slots=None):
        """Returns (routed, shared, shared_gate) like model.py:490-518."""
        layer = layer_view(layer)
        E = layer.experts.w13_weight.shape[0]
        # the bias enters before the bf16 rounding of the logits, as in moe()
        bias = getattr(layer, "router_bias", None)
        if bias is not None:
            bias = bias.to(torch.float32).contiguous()
        logits = ops.router_logits(x, layer.router_weight, bias)
        router, shared_gate = logits[:, :E], logits[:, E:E + 1]
        slots, start = self._padding(row_slots)
        weights, ids = ops.route_topk(router, self.top_k, row_slots=slots, padding_start=start)
        routed, shared = ops.moe_experts(x, ids, weights, layer.experts, layer.shared_expert,
                                         workspace=self._workspace(len(x), layer))
        return routed, shared, shared_gate

    def routed_moe(self, x, router, experts, decode, *, row_slots=None):
        """Routed experts from given router logits (model.py:520-583)."""
        slots, start = self._padding(row_slots)
        weights, ids = ops.route_topk(router, self.top_k, weights_dtype=torch.bfloat16,
                                      row_slots=slots, padding_start=start)
        routed, _ = ops.moe_experts(x, ids, weights, experts)
        return routed
