"""Operator-level drop-ins for src/drama3/kernels.py (MoE hot path only).

Signatures follow the reference so a caller swaps the import:
  route(logits)                                   kernels.py:379-383
  small_batch_moe(x, ids, weights, experts, ...)  kernels.py:325-357
  native_moe(x, ids, weights, experts, ...)       kernels.py:702-779
  silu_mul(projected)                             kernels.py:396-402
  combine_experts(routed, shared, gate)           kernels.py:442-445
  linear(x, weight)                               kernels.py:274-287
The reference's tile knobs (up_rows, down_rows, down_warps, block_m, group_m,
atomic) are accepted for call compatibility; the B200 kernels choose their own
tiling (weight-streaming engine for few tokens per expert).
"""

from __future__ import annotations

import torch

from . import experimental_fp8, ops


def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """y [M, N] = x [M, K] . weight [N, K]^T (kernels.py:274-287).

    The reference dispatches its BF16 projections to a Triton GEMV (M = 1),
    FlashInfer's mm_bf16 (2 <= M <= 32) or F.linear. Here every projection is
    the weight-only FP8 GEMV with 128x128 block scales, the dense FP8
    projection of this path: a weight is quantised once, on its first use
    (experimental_fp8.register, keyed by data_ptr like the reference's
    WEIGHTS table), and every later call reuses it. Activations stay bf16
    and the sums fp32, for any M."""
    if weight.data_ptr() not in experimental_fp8.WEIGHTS:
        experimental_fp8.register(weight)
    return experimental_fp8.linear(x, weight)


def route(logits: torch.Tensor, k: int = 8):
    """fp32 softmax, top-k (ties to the lower expert id), renormalised weights
    in the logits dtype. Returns (weights, indices int64)."""
    return ops.route_topk(logits, k)


def small_batch_moe(x, topk_ids, topk_weights, experts, up_rows=4, down_rows=4, down_warps=8):
    """Routed experts for a decode batch; bf16 [T, H]."""
    for name, v in (("up_rows", up_rows), ("down_rows", down_rows), ("down_warps", down_warps)):
        if int(v) <= 0:
            raise ValueError(f"{name} must be positive")
    routed, _ = ops.moe_experts(x, topk_ids.contiguous(), topk_weights, experts)
    return routed


def native_moe(x, topk_ids, topk_weights, experts, block_m=16, group_m=1, atomic=False):
    """Routed experts for any batch; bf16 [T, H]. The per-pair down outputs
    are combined in fixed rank order in fp32 (the non-atomic reference form,
    kernels.py:764-779), so `atomic` selects nothing different."""
    if block_m not in (16, 32, 64, 128) or group_m <= 0:
        raise ValueError("block_m must be 16, 32, 64 or 128 and group_m positive")
    routed, _ = ops.moe_experts(x, topk_ids.contiguous(), topk_weights, experts)
    return routed


def silu_mul(projected: torch.Tensor) -> torch.Tensor:
    return ops.silu_mul(projected)


def combine_experts(routed, shared, gate):
    return ops.combine_experts(routed, shared, gate)


def add_norm(x, residual, weight, epsilon):
    """kernels.py:418-423: mutates `residual`, returns the normalised rows."""
    return ops.add_norm(x, residual, weight, epsilon)


def combine_experts_add_norm(routed, shared, gate, residual, weight, epsilon):
    """kernels.py:483-499: mutates `residual`, returns the normalised rows."""
    return ops.combine_experts_add_norm(routed, shared, gate, residual, weight, epsilon)


def combine_experts_add_norm_inverse(routed, shared, gate, inverse, residual, weight, epsilon):
    """kernels.py:540-556: compact routed/shared rows gathered by `inverse`."""
    return ops.combine_experts_add_norm(routed, shared, gate, residual, weight, epsilon, inverse=inverse)


def moe_permute(topk_ids: torch.Tensor, num_experts: int, block_m: int = 16):
    """The device bucketing of native_moe (kernels.py:711-731):
    (counts, starts, total, sorted_ids, expert_ids)."""
    counts, starts, total, sorted_ids, expert_ids, *_ = ops.moe_permute(topk_ids, num_experts, block_m)
    return counts, starts, total, sorted_ids, expert_ids


def quantize_groups(x: torch.Tensor):
    """Activation FP8 quantisation per 1x128 group (Fish quantize_groups):
    (q e4m3 [T,H], scales f32 [T,H/128])."""
    return ops.quant_act_fp8(x, transposed=False)
