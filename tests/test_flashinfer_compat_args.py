"""Host-side argument contract of the FlashInfer-compatible entry: arguments
outside what the reference passes (src/drama3/model.py:556-580) raise before any
device work instead of running a different algorithm."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from d3moe.flashinfer_compat import RoutingMethodType, WeightLayout, trtllm_fp8_block_scale_moe  # noqa: E402

E, I, H, T = 8, 128, 256, 4


def args(**over):
    a = dict(
        routing_logits=torch.zeros(T, E), routing_bias=None,
        hidden_states=torch.zeros(T, H, dtype=torch.float8_e4m3fn),
        hidden_states_scale=torch.ones(H // 128, T),
        gemm1_weights=torch.zeros(E, 2 * I, H, dtype=torch.float8_e4m3fn),
        gemm1_weights_scale=torch.ones(E, 2 * I // 128, H // 128),
        gemm2_weights=torch.zeros(E, H, I, dtype=torch.float8_e4m3fn),
        gemm2_weights_scale=torch.ones(E, H // 128, I // 128),
        num_experts=E, top_k=2, n_group=None, topk_group=None, intermediate_size=I,
        local_expert_offset=0, local_num_experts=E, routed_scaling_factor=1.0,
        routing_method_type=RoutingMethodType.RenormalizeNaive, use_shuffled_weight=False,
        weight_layout=WeightLayout.MajorK)
    a.update(over)
    return a


@pytest.mark.parametrize("over", [
    dict(routing_method_type=RoutingMethodType.DeepSeekV3),
    dict(routing_method_type=RoutingMethodType.Renormalize),
    dict(n_group=4, topk_group=2),
    dict(use_shuffled_weight=True),  # shuffled bytes need the BlockMajorK tag
    dict(weight_layout=WeightLayout.BlockMajorK),  # and the tag needs shuffled bytes
    dict(weight_layout=WeightLayout.MajorMn),
    dict(routed_scaling_factor=2.5),
    dict(do_finalize=False),
    dict(activation_type=4),
])
def test_unsupported_arguments_raise(over):
    with pytest.raises(NotImplementedError):
        trtllm_fp8_block_scale_moe(**args(**over))


@pytest.mark.parametrize("over", [
    dict(num_experts=16),
    dict(intermediate_size=256),
    dict(local_num_experts=4),
    dict(local_expert_offset=1),
    dict(hidden_states=torch.zeros(T + 1, H, dtype=torch.float8_e4m3fn)),
])
def test_inconsistent_shapes_raise(over):
    with pytest.raises(ValueError):
        trtllm_fp8_block_scale_moe(**args(**over))


def test_block_major_k_unshuffle_inverts_the_reference_shuffle():
    """BlockMajorK weights (the reference's blocked_moe_weight, model.py:41-52,
    restated here: K blocks to the front, rows permuted by FlashInfer's 64-row
    epilogue map) come back to the MajorK bytes exactly, from the 4-D shape the
    shuffle returns and from the same bytes viewed [E, rows, K]."""
    pytest.importorskip("flashinfer")
    from flashinfer.utils import get_shuffle_matrix_a_row_indices

    from d3moe.flashinfer_compat import unshuffle_block_major_k

    g = torch.Generator().manual_seed(0)
    for E_, rows, K in ((2, 256, 384), (3, 1536, 2048)):
        w = torch.randint(0, 256, (E_, rows, K), generator=g, dtype=torch.uint8)
        order = get_shuffle_matrix_a_row_indices(w[0], 64)
        blocked = w.view(E_, rows, K // 128, 128).permute(0, 2, 1, 3)[:, :, order, :].contiguous()
        for shaped in (blocked, blocked.view(E_, rows, K)):
            back = unshuffle_block_major_k(shaped.view(torch.float8_e4m3fn))
            assert back.shape == (E_, rows, K)
            assert torch.equal(back.view(torch.uint8), w)


def test_block_major_k_cache_follows_in_place_writes():
    """The un-shuffled copy is cached per weight tensor; writing the weights in
    place (through any view) must not return the stale copy, and the cache
    keeps its input alive so that no other tensor can take its address."""
    pytest.importorskip("flashinfer")
    from flashinfer.utils import get_shuffle_matrix_a_row_indices

    from d3moe import flashinfer_compat as fc

    g = torch.Generator().manual_seed(1)
    E_, rows, K = 2, 256, 256
    w = torch.randint(0, 256, (E_, rows, K), generator=g, dtype=torch.uint8)
    order = get_shuffle_matrix_a_row_indices(w[0], 64)

    def shuffle(m):
        return m.view(E_, rows, K // 128, 128).permute(0, 2, 1, 3)[:, :, order, :].contiguous()

    blocked = shuffle(w).view(torch.float8_e4m3fn)
    first = fc.unshuffle_block_major_k(blocked)
    assert fc.unshuffle_block_major_k(blocked) is first  # cached
    w2 = torch.randint(0, 256, (E_, rows, K), generator=g, dtype=torch.uint8)
    blocked.view(torch.uint8).copy_(shuffle(w2))  # in place, through a view
    again = fc.unshuffle_block_major_k(blocked)
    assert again is not first
    assert torch.equal(again.view(torch.uint8), w2)
    key = (blocked.data_ptr(), tuple(blocked.shape), blocked.dtype)
    assert fc._unshuffled[key][0] is blocked
