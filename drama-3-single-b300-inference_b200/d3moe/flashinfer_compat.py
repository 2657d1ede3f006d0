"""Drop-in for FlashInfer's `trtllm_fp8_block_scale_moe`, the call the reference
makes for decode batches above 8 rows and for FlashInfer prefill
(src/drama3/model.py:544-583).

The reference prepares FlashInfer's operands once per layer: w13 rows
reordered to [up | gate] with their scale rows (model.py:196-201), hidden
states quantised per 1x128 group with the scales transposed to [H/128, T]
(moe_input.py:28-30), fp32 router logits. This function takes exactly those
operands and runs them on this library's kernels: RenormalizeNaive routing
(softmax over all experts, top-k, renormalise; routing_method_type=4), the
[up | gate] weights read in place (no copy), FP8 gate_up with SiLU*mul and
requantisation, FP8 down and the fixed-order routed combine. Arguments outside
what the reference passes raise instead of running a different algorithm.

Weights in FlashInfer's BlockMajorK layout (use_shuffled_weight=True,
weight_layout=BlockMajorK: what the reference passes when
DRAMA3_MOE_LAYOUT=blocked, model.py:152, 203-206, 574-576, shuffled by
blocked_moe_weight, model.py:41-52) are brought back to the MajorK
checkpoint layout once per weight tensor (a copy, cached per input tensor
until that tensor is written in place) and then run like MajorK weights.
The shuffle moves 128-byte K blocks to the
front ([E, K/128, rows, 128]) and permutes the rows inside each K block by
FlashInfer's epilogue row map for a 64-row tile
(flashinfer.utils.get_shuffle_matrix_a_row_indices); the scales keep their
logical order.
"""

from __future__ import annotations

import torch

from . import ops


class WeightLayout:
    """FlashInfer's weight layout tags (flashinfer.fused_moe.WeightLayout)."""

    MajorK = 0
    MajorMn = 1
    BlockMajorK = 2


class RoutingMethodType:
    """FlashInfer's routing method tags (the ones the reference can reach)."""

    Default = 0
    Renormalize = 1
    DeepSeekV3 = 2
    Llama4 = 3
    RenormalizeNaive = 4


_views: dict = {}
_unshuffled: dict = {}


def unshuffle_block_major_k(weight: torch.Tensor) -> torch.Tensor:
    """Inverse of the reference's blocked_moe_weight (model.py:41-52): e4m3
    [E, K/128, rows, 128] (the shape blocked_moe_weight returns) or the same
    bytes as [E, rows, K] -> the MajorK tensor [E, rows, K] it was made from.
    Cached per input (address, shape, dtype). The entry holds a reference to
    the input, so no other tensor can take its address while it is cached,
    and the input's version counter, so an in-place write to the weights (or
    to any view of them) makes the next call un-shuffle again."""
    key = (weight.data_ptr(), tuple(weight.shape), weight.dtype)
    hit = _unshuffled.get(key)
    if hit is not None and hit[1] == weight._version:
        return hit[2]
    from flashinfer.utils import get_shuffle_matrix_a_row_indices

    if weight.dim() == 4:
        E, KB, rows, last = weight.shape
        if last != 128:
            raise ValueError("BlockMajorK weights are [E, K/128, rows, 128]")
        K = KB * 128
    else:
        E, rows, K = weight.shape
        if K % 128:
            raise ValueError("BlockMajorK weights need K a multiple of 128")
    order = get_shuffle_matrix_a_row_indices(torch.empty((rows, K), dtype=torch.uint8), 64)
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(rows, dtype=order.dtype)
    blocks = weight.view(torch.uint8).reshape(E, K // 128, rows, 128)
    out = blocks[:, :, inverse.to(weight.device), :].permute(0, 2, 1, 3).contiguous()
    out = out.view(E, rows, K).view(weight.dtype)
    _unshuffled[key] = (weight, weight._version, out)
    return out


def _expert_view(w13, s13, w2, s2) -> ops.ExpertView:
    key = (w13.data_ptr(), s13.data_ptr(), w2.data_ptr(), s2.data_ptr(), tuple(w13.shape), tuple(w2.shape))
    view = _views.get(key)
    if view is None:
        view = ops.ExpertView(tensors=(w13, s13, w2, s2), gate_up_order="up_gate")
        _views[key] = view
    return view


def trtllm_fp8_block_scale_moe(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                               gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                               num_experts, top_k, n_group, topk_group, intermediate_size,
                               local_expert_offset, local_num_experts, routed_scaling_factor,
                               routing_method_type=0, use_shuffled_weight=False,
                               weight_layout=WeightLayout.MajorK, do_finalize=True, enable_pdl=None,
                               tune_max_num_tokens=8192, activation_type=3, **unused):
    """Routed MoE output bf16 [T, H] (model.py:556-581 arguments).

    routing_logits f32 (or bf16) [T, num_experts]; routing_bias [num_experts] or
    None; hidden_states e4m3 [T, H]; hidden_states_scale f32 [H/128, T];
    gemm1_weights e4m3 [local_num_experts, 2*intermediate_size, H] in [up | gate]
    row order with scales [.., 2I/128, H/128]; gemm2_weights e4m3 [.., H, I] with
    scales [.., H/128, I/128]. Experts outside [local_expert_offset,
    local_expert_offset + local_num_experts) contribute nothing."""
    if routing_method_type != RoutingMethodType.RenormalizeNaive:
        raise NotImplementedError("only routing_method_type=4 (RenormalizeNaive) is implemented")
    if n_group or topk_group:
        raise NotImplementedError("grouped top-k routing (n_group/topk_group) is not implemented")
    if use_shuffled_weight != (weight_layout == WeightLayout.BlockMajorK) or weight_layout == WeightLayout.MajorMn:
        raise NotImplementedError("weights must be MajorK (unshuffled) or BlockMajorK with "
                                  "use_shuffled_weight=True, the two layouts the reference passes")
    if weight_layout == WeightLayout.BlockMajorK:
        gemm1_weights = unshuffle_block_major_k(gemm1_weights)
        gemm2_weights = unshuffle_block_major_k(gemm2_weights)
    if routed_scaling_factor not in (None, 1.0):
        raise NotImplementedError("routed_scaling_factor other than 1.0 is not implemented")
    if not do_finalize:
        raise NotImplementedError("do_finalize=False (unfinalised GEMM2 output) is not implemented")
    if activation_type not in (None, 3):
        raise NotImplementedError("only the SwiGLU activation (activation_type=3) is implemented")
    T, E_all = routing_logits.shape
    if E_all != num_experts:
        raise ValueError(f"routing_logits has {E_all} experts, num_experts={num_experts}")
    E_local, rows, H = gemm1_weights.shape
    if E_local != local_num_experts or rows != 2 * intermediate_size:
        raise ValueError("gemm1_weights must be [local_num_experts, 2*intermediate_size, H]")
    if not 0 <= local_expert_offset <= num_experts - local_num_experts:
        raise ValueError("local experts must lie inside [0, num_experts)")
    if tuple(hidden_states.shape) != (T, H):
        raise ValueError("hidden_states must be [T, H]")
    view = _expert_view(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    weights, ids = ops.route_topk(routing_logits.contiguous(), top_k, bias=routing_bias,
                                  weights_dtype=torch.bfloat16)
    if local_expert_offset:
        ids = ids - local_expert_offset
    return ops.moe_experts_fp8(hidden_states, hidden_states_scale, ids, weights, view, transposed=True)
