"""GPU parity of the FlashInfer-compatible entry: trtllm_fp8_block_scale_moe's
operands (fp32 logits, e4m3 hidden states with [H/128, T] scales, w13 in
[up | gate] order; src/drama3/model.py:196-201, 544-581) run on this library's
kernels. Routing is bit-exact against the oracle, values within the layer
tolerance; the [up | gate] weights read in place give the [gate | up] result bit
for bit, and pre-quantised input gives the bf16-input path's result bit for
bit."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import assert_close, experts_to_oracle, fp8_bytes, to_bf16  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

E, I, H, K = 128, 768, 2048, 8


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth
    lw = synth.make_layer(E, I, H, seed=41, device="cuda")
    ex = lw.experts
    gate, up = ex.w13_weight.chunk(2, dim=1)
    gs, us = ex.w13_scale_inv.chunk(2, dim=1)
    fi = (torch.cat((up, gate), dim=1).contiguous(), torch.cat((us, gs), dim=1).contiguous(),
          ex.w2_weight, ex.w2_scale_inv)
    return lw, fi, experts_to_oracle(ex)


def inputs(T, n_logits, seed):
    from d3moe import ops
    rng = np.random.default_rng(seed)
    x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    q, s = ops.quant_act_fp8(to_bf16(x), transposed=True)
    logits = torch.from_numpy(rng.standard_normal((T, n_logits)).astype(np.float32) * 2.0).cuda()
    return x, q, s, logits


def call(logits, bias, q, s, fi, n_experts, offset=0):
    from d3moe.flashinfer_compat import trtllm_fp8_block_scale_moe
    return trtllm_fp8_block_scale_moe(
        routing_logits=logits, routing_bias=bias, hidden_states=q, hidden_states_scale=s,
        gemm1_weights=fi[0], gemm1_weights_scale=fi[1], gemm2_weights=fi[2], gemm2_weights_scale=fi[3],
        num_experts=n_experts, top_k=K, n_group=None, topk_group=None, intermediate_size=I,
        local_expert_offset=offset, local_num_experts=fi[0].shape[0], routed_scaling_factor=1.0,
        routing_method_type=4, use_shuffled_weight=False, weight_layout=0, tune_max_num_tokens=4096,
        enable_pdl=True)


@pytest.mark.parametrize("T,with_bias,prefill", [(16, False, False), (64, True, False), (300, False, True)])
def test_matches_oracle(layer, T, with_bias, prefill):
    from d3moe import ops
    lw, fi, ex = layer
    _, q, s, logits = inputs(T, E, seed=T)
    bias = torch.randn(E, generator=torch.Generator().manual_seed(T)).cuda() if with_bias else None
    with ops.prefill_min_tokens(1 if prefill else 1 << 30):
        out = call(logits, bias, q, s, fi, E)
        _, ids = ops.route_topk(logits, K, bias=bias, weights_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    bias_np = None if bias is None else bias.cpu().numpy()
    w_o, ids_o = O.route(logits.cpu().numpy(), K, bias=bias_np)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    ref = O.moe_experts_q(fp8_bytes(q), s.cpu().numpy().T, ids_o, O.bf16_round(w_o), ex,
                          rows_bf16=prefill)
    assert_close(out.float().cpu().numpy(), ref, what=f"flashinfer-compatible T={T}")


@pytest.mark.parametrize("T", [64, 1344])
def test_up_gate_and_prequant_match_the_native_paths(layer, T):
    from d3moe import ops
    lw, fi, _ = layer
    x, q, s, logits = inputs(T, E, seed=7 + T)
    w, ids = ops.route_topk(logits, K, weights_dtype=torch.bfloat16)
    native = ops.ExpertView(lw.experts)
    swapped = ops.ExpertView(tensors=fi, gate_up_order="up_gate")
    a = ops.moe_experts_fp8(q, s, ids, w, swapped)
    b = ops.moe_experts_fp8(q, s, ids, w, native)
    c, _ = ops.moe_experts(to_bf16(x), ids, w, native)
    # [T, H/128] scales give the same result as the transposed layout
    d = ops.moe_experts_fp8(q, s.t().contiguous(), ids, w, native, transposed=False)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(b, c)
    assert torch.equal(b, d)


def test_local_expert_offset(layer):
    """The layer's 128 experts as experts 128..255 of a 256-expert router:
    picks outside the local range contribute nothing."""
    from d3moe import ops
    lw, fi, ex = layer
    T = 64
    _, q, s, logits = inputs(T, 2 * E, seed=99)
    out = call(logits, None, q, s, fi, 2 * E, offset=E)
    _, ids = ops.route_topk(logits, K, weights_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    w_o, ids_o = O.route(logits.cpu().numpy(), K)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    local = ids_o - E
    assert ((local >= 0) & (local < E)).any() and ((local < 0) | (local >= E)).any()
    ref = O.moe_experts_q(fp8_bytes(q), s.cpu().numpy().T, local, O.bf16_round(w_o), ex)
    assert_close(out.float().cpu().numpy(), ref, what="local experts")


def test_block_major_k_weights_give_the_major_k_result(layer):
    """Weights shuffled into FlashInfer's BlockMajorK layout the way the
    reference does it (blocked_moe_weight, model.py:41-52, restated: K blocks
    first, rows permuted by FlashInfer's 64-row epilogue map), passed with
    use_shuffled_weight=True and weight_layout=BlockMajorK, give the MajorK
    call's output bit for bit."""
    pytest.importorskip("flashinfer")
    from flashinfer.utils import get_shuffle_matrix_a_row_indices

    from d3moe.flashinfer_compat import WeightLayout, trtllm_fp8_block_scale_moe

    lw, fi, _ = layer
    _, q, s, logits = inputs(64, E, seed=5)

    def blocked(w):
        e_, rows, k_ = w.shape
        order = get_shuffle_matrix_a_row_indices(w[0].view(torch.uint8).cpu(), 64).to(w.device)
        b = w.view(torch.uint8).view(e_, rows, k_ // 128, 128).permute(0, 2, 1, 3)[:, :, order, :]
        return b.contiguous().view(w.dtype)

    ref = call(logits, None, q, s, fi, E)
    out = trtllm_fp8_block_scale_moe(
        routing_logits=logits, routing_bias=None, hidden_states=q, hidden_states_scale=s,
        gemm1_weights=blocked(fi[0]), gemm1_weights_scale=fi[1], gemm2_weights=blocked(fi[2]),
        gemm2_weights_scale=fi[3], num_experts=E, top_k=K, n_group=None, topk_group=None,
        intermediate_size=I, local_expert_offset=0, local_num_experts=E, routed_scaling_factor=1.0,
        routing_method_type=4, use_shuffled_weight=True, weight_layout=WeightLayout.BlockMajorK,
        tune_max_num_tokens=4096, enable_pdl=True)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
