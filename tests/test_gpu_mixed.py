"""GPU parity of the mixed decode + packed-prefill MoE call
(src/drama3/mixed_model.py:193-246): decode rows first, then packed prompts
and their padding; the MoE runs on the compact rows `keep` of a row-reuse plan,
padding rows route with row 0's logits, and the fused exit scatters back
through `inverse`. Routing is bit-exact against the oracle; values hold the
layer tolerance; the reuse call equals the full-row call and the reference's
two-step sequence bit for bit."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import experts_to_oracle, from_bf16, rel_l2, to_bf16  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

E, I, H, K = 128, 768, 2048, 8
PAD = 512  # reserved-slot boundary (the reference's slots // 2)


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth
    lw = synth.make_layer(E, I, H, seed=33, device="cuda")
    return lw, experts_to_oracle(lw.experts), experts_to_oracle(lw.shared)


def prompt(length, value):
    p = torch.zeros((length, 11), dtype=torch.int64)
    p[:, 0] = value
    p[:, 1] = torch.arange(length)
    return p


def layout(decode_rows, decode_pad, prompts, capacity, buckets, seed):
    """x [full, H] with aliased rows equal to their owners, the row slots, and
    the plan. The last `decode_pad` decode rows and the trailing prompt padding
    carry reserved slots."""
    from d3moe import mixed
    plan = mixed.plan_row_reuse(prompts, decode_rows, capacity, buckets)
    assert plan is not None
    full = decode_rows + capacity
    dslots = list(range(decode_rows - decode_pad)) + [PAD + 1 + i for i in range(decode_pad)]
    seq_slots = [100 + i for i in range(len(prompts))] + [PAD + 100]
    slots = mixed.packed_row_slots(dslots, [len(p) for p in prompts], seq_slots, capacity)
    rng = np.random.default_rng(seed)
    x = O.bf16_round(rng.standard_normal((full, H)).astype(np.float32))
    owner = plan.keep.numpy()[plan.inverse.numpy()]
    x = x[owner]  # an aliased row holds its owner's hidden state
    return x, slots, plan


def small_layout():
    a = prompt(200, 1)
    b = a[:100].clone()
    b[90:, 2] = 5  # b repeats a's first 90 rows
    return layout(16, 2, [a, a.clone(), b], 512, (256,), seed=4)


def full_layout():
    """M = 64 + 1280 = 1344 rows (the reference's D64/P1280 mixed graph) with 6
    prompts; 256-aligned compact bucket 1088."""
    base = prompt(256, 2)
    prompts = [base, base.clone(), base[:200].clone(), prompt(180, 3), prompt(150, 4),
               base[:120].clone()]
    prompts[2][150:, 4] = 9
    return layout(64, 6, prompts, 1280, (1088,), seed=8)


def run_fused(ops, lw, x, slots, plan, res, nw, reuse=True, status=None):
    xt = to_bf16(x)
    rt = to_bf16(res)
    kw = {}
    if reuse:
        keep, inv = plan.keep.cuda(), plan.inverse.cuda()
        kw = dict(keep=keep, inverse=inv, row_slots=torch.from_numpy(slots).cuda()[keep],
                  padding_start=PAD)
    else:
        kw = dict(row_slots=torch.from_numpy(slots).cuda(), padding_start=PAD)
    out, ids, w = ops.moe_layer(xt, lw.router, lw.experts, lw.shared, K, residual=rt,
                                norm_weight=to_bf16(nw), return_routing=True, status=status, **kw)
    return out, rt, ids, w


def within(actual, expected, what):
    a = np.asarray(actual, np.float64)
    ulp = np.spacing(np.abs(expected).astype(np.float32)).astype(np.float64) * 65536.0
    assert (np.abs(a - expected) <= 2e-2 + ulp).all(), what
    assert rel_l2(a, expected) <= 1e-2, what


@pytest.mark.parametrize("prefill", [False, True])
def test_mixed_layer_matches_oracle(layer, prefill):
    from d3moe import ops
    lw, ex, sh = layer
    x, slots, plan = small_layout()
    full = len(x)
    rng = np.random.default_rng(6)
    res0 = O.bf16_round((rng.standard_normal((full, H)) * 2.0).astype(np.float32))
    nw = O.bf16_round((rng.standard_normal(H) * 0.1).astype(np.float32))
    with ops.prefill_min_tokens(1 if prefill else 1 << 30):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        out, rt, ids, _ = run_fused(ops, lw, x, slots, plan, res0, nw, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    keep, inv = plan.keep.numpy(), plan.inverse.numpy()
    out_o, res_o, ids_o, _ = O.moe_layer_rows(x, from_bf16(lw.router), ex, sh, res0, nw, 1e-6, K,
                                              keep=keep, inverse=inv, row_slots=slots[keep],
                                              padding_start=PAD, rows_bf16=prefill)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    within(from_bf16(rt), res_o, "residual")
    within(from_bf16(out), out_o, "out")


def test_padding_rows_route_like_row_zero(layer):
    from d3moe import ops
    lw, _, _ = layer
    x, slots, plan = full_layout()
    res0 = np.zeros((len(x), H), np.float32)
    nw = np.zeros(H, np.float32)
    _, _, ids, w = run_fused(ops, lw, x, slots, plan, res0, nw)
    keep = plan.keep.numpy()
    pad = slots[keep] >= PAD
    assert pad.sum() > 0 and not pad[0]
    ids, w = ids.cpu(), w.cpu()
    assert torch.equal(ids[torch.from_numpy(pad)], ids[0:1].expand(int(pad.sum()), K))
    assert torch.equal(w[torch.from_numpy(pad)], w[0:1].expand(int(pad.sum()), K))
    assert not torch.equal(ids[~torch.from_numpy(pad)], ids[0:1].expand(int((~pad).sum()), K))


@pytest.mark.parametrize("prefill", [False, True])
def test_row_reuse_equals_full_rows(layer, prefill):
    """Running the MoE once per owner and gathering through `inverse` gives the
    full-row call's residual and output bit for bit."""
    from d3moe import ops
    lw, _, _ = layer
    x, slots, plan = full_layout()
    rng = np.random.default_rng(12)
    res0 = O.bf16_round((rng.standard_normal((len(x), H)) * 2.0).astype(np.float32))
    nw = O.bf16_round((rng.standard_normal(H) * 0.1).astype(np.float32))
    with ops.prefill_min_tokens(1 if prefill else 1 << 30):
        out_r, res_r, _, _ = run_fused(ops, lw, x, slots, plan, res0, nw, reuse=True)
        out_f, res_f, _, _ = run_fused(ops, lw, x, slots, plan, res0, nw, reuse=False)
    torch.cuda.synchronize()
    assert torch.equal(res_r, res_f)
    assert torch.equal(out_r, out_f)


def test_fused_matches_two_step(layer):
    """One call == normalized.index_select(0, keep) -> moe_parts(row_slots) ->
    combine_experts_add_norm_inverse (mixed_model.py:200-246)."""
    from d3moe import kernels, ops
    from d3moe.model import MoE
    lw, _, _ = layer
    x, slots, plan = full_layout()
    rng = np.random.default_rng(13)
    res0 = O.bf16_round((rng.standard_normal((len(x), H)) * 2.0).astype(np.float32))
    nw = O.bf16_round((rng.standard_normal(H) * 0.1).astype(np.float32))

    class L:
        experts = lw.experts
        shared_expert = lw.shared
        router_weight = lw.router

    moe = MoE(padding_start=PAD)
    keep, inv = plan.keep.cuda(), plan.inverse.cuda()
    xt = to_bf16(x)
    compact_slots = torch.from_numpy(slots).cuda().index_select(0, keep)
    r_fused = to_bf16(res0)
    out_fused = moe.moe_add_norm(xt, L, r_fused, to_bf16(nw), 1e-6, keep=keep, inverse=inv,
                                 row_slots=compact_slots)
    parts = moe.moe_parts(xt.index_select(0, keep), L, decode=True, row_slots=compact_slots)
    r_two = to_bf16(res0)
    out_two = kernels.combine_experts_add_norm_inverse(*parts, inv, r_two, to_bf16(nw), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(r_fused, r_two)
    assert torch.equal(out_fused, out_two)


def test_bad_row_maps_set_the_status_word(layer):
    """A keep or inverse value outside its tensor is reported in the status word
    (D3_STATUS_BAD_ROW) and row 0 is read in its place; no access leaves the
    tensors."""
    from d3moe import ops
    lw, _, _ = layer
    T, full = 64, 80
    rng = np.random.default_rng(2)
    xt = to_bf16(O.bf16_round(rng.standard_normal((full, H)).astype(np.float32)))
    res = torch.zeros((full, H), dtype=torch.bfloat16, device="cuda")
    nw = torch.zeros(H, dtype=torch.bfloat16, device="cuda")
    keep = torch.arange(T, dtype=torch.int64, device="cuda")
    inv = torch.arange(full, dtype=torch.int64, device="cuda") % T
    for what in ("keep", "inverse"):
        k2, i2 = keep.clone(), inv.clone()
        if what == "keep":
            k2[5] = full
        else:
            i2[7] = -1
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        ops.moe_layer(xt, lw.router, lw.experts, lw.shared, K, residual=res.clone(), norm_weight=nw,
                      keep=k2, inverse=i2, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 2, what
