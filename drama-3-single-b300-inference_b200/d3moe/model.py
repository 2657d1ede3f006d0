"""Model-level MoE entry points with the reference's signatures
(DramaModel.moe / moe_parts / routed_moe, src/drama3/model.py:485-583).

`layer` is any object with:
  experts                   routed expert container (w13_weight, ...)
  shared_expert             shared expert container (E = 1 or unbatched)
  router_weight             bf16 [E+1, H]: router rows + shared-expert gate row
  router_bias (optional)    f32 [E], added to the router logits

Routing always runs on the device (route_topk); the routed and shared experts
run in the same launches of the expert engine. No host synchronisation, so a
decode step built from these calls is CUDA-graph capturable.
"""

from __future__ import annotations

import torch

from . import ops


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
        slots, start = self._padding(row_slots)
        T = len(keep) if keep is not None else len(x)
        return ops.moe_layer(x, layer.router_weight, layer.experts, layer.shared_expert, self.top_k,
                             router_bias=getattr(layer, "router_bias", None),
                             workspace=self._workspace(T, layer), residual=residual,
                             norm_weight=norm_weight, norm_eps=eps, keep=keep, inverse=inverse,
                             row_slots=slots, padding_start=start)

    def moe_parts(self, x: torch.Tensor, layer, decode: bool = False, *, row_slots=None):
        """Returns (routed, shared, shared_gate) like model.py:490-518."""
        E = layer.experts.w13_weight.shape[0]
        logits = ops.router_logits(x, layer.router_weight)
        router, shared_gate = logits[:, :E], logits[:, E:E + 1]
        bias = getattr(layer, "router_bias", None)
        slots, start = self._padding(row_slots)
        weights, ids = ops.route_topk(router, self.top_k, bias=bias, row_slots=slots,
                                      padding_start=start)
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
