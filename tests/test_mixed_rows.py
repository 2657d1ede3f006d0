"""Host logic of the mixed decode + packed-prefill call: the row-reuse plan
(the contract of src/drama3/row_reuse.py:45-105, exercised like
tests/test_row_reuse.py of the reference), the per-row slots, and the oracle's
padding-router rule."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from d3moe import mixed  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402


def prompt(length, value=0):
    p = torch.zeros((length, 11), dtype=torch.int64)
    p[:, 0] = value
    return p


def verify_plan(plan, prompts):
    """Every full row maps to a compact row whose owner is the same position of
    an earlier (or the same) prompt with an identical causal prefix; decode and
    padding rows own themselves; spare compact rows repeat row 0."""
    d = plan.decode_rows
    full = d + plan.prefill_capacity
    keep, inverse = plan.keep.numpy(), plan.inverse.numpy()
    assert len(keep) == plan.compact_rows and len(inverse) == full
    assert inverse.min() >= 0 and inverse.max() < plan.compact_rows
    owner = keep[inverse]
    starts = np.cumsum([d] + [len(p) for p in prompts])
    assert (owner[:d] == np.arange(d)).all()
    assert (owner[starts[-1]:] == np.arange(starts[-1], full)).all()
    for s, p in enumerate(prompts):
        for pos in range(len(p)):
            row = starts[s] + pos
            src = int(owner[row])
            assert d <= src <= row
            prev = int(np.searchsorted(starts, src, side="right") - 1)
            assert src - starts[prev] == pos
            assert torch.equal(p[:pos + 1], prompts[prev][:pos + 1])
    assert len(np.unique(owner)) == plan.unique_rows
    assert (keep[:plan.unique_rows] == np.flatnonzero(owner == np.arange(full))).all()
    assert (keep[plan.unique_rows:] == 0).all()


@pytest.mark.parametrize("d,capacity,span,compact", mixed.MIXED_ROW_REUSE_BUCKETS)
def test_bucket_shapes(d, capacity, span, compact):
    sizes = [capacity // 9] * 8
    prompts = [prompt(n, 3) for n in sizes]
    plan = mixed.plan_row_reuse(prompts, d, capacity, (compact,))
    assert plan is not None and plan.compact_rows == compact
    assert max(sizes + [capacity - sum(sizes)]) <= span
    verify_plan(plan, prompts)
    assert plan.matches_prompts(prompts)
    changed = [p.clone() for p in prompts]
    changed[3][5, 2] = 1
    assert not plan.matches_prompts(changed)


@pytest.mark.parametrize("column", range(11))
def test_a_changed_column_stops_the_alias(column):
    a, b = prompt(128), prompt(128)
    b[17, column] = 7
    prompts = [a, b, a.clone(), b.clone()]
    plan = mixed.plan_row_reuse(prompts, 64, 768, (576,))
    assert plan is not None
    verify_plan(plan, prompts)
    inv = plan.inverse
    assert torch.equal(inv[64:81], inv[192:209])
    assert torch.all(inv[81:192] != inv[209:320])


def test_partial_prefixes_and_order():
    a, b = prompt(128), prompt(128)
    b[12, 10] = 1
    prompts = [a, b, a[:80], b[:100], a.clone()]
    plan = mixed.plan_row_reuse(prompts, 64, 768, (576,))
    assert plan is not None
    verify_plan(plan, prompts)
    rev = list(reversed(prompts))
    plan_r = mixed.plan_row_reuse(rev, 64, 768, (576,))
    assert plan_r is not None
    verify_plan(plan_r, rev)
    assert not torch.equal(plan.packed_indices, plan_r.packed_indices)
    survivors = [a, a.clone(), a.clone()]
    assert mixed.plan_row_reuse(survivors, 64, 768, (576,)) is not None
    assert mixed.plan_row_reuse(survivors[:2], 64, 768, (576,)) is None


def test_no_alias_or_no_bucket():
    distinct = [prompt(128, i) for i in range(6)]
    assert mixed.plan_row_reuse(distinct, 64, 768, (576,)) is None
    assert mixed.plan_row_reuse(distinct, 64, 768, ()) is None
    assert mixed.plan_row_reuse([prompt(3)] * 8, 64, 768, (576,)) is None


def test_smallest_bucket_that_fits():
    prompts = [prompt(180), prompt(180), prompt(170, 1), prompt(170, 1)]
    plan = mixed.plan_row_reuse(prompts, 64, 1536, (1344, 1088))
    assert plan is not None and plan.compact_rows == 1344
    assert -(-plan.unique_rows // 64) * 64 <= plan.compact_rows
    verify_plan(plan, prompts)


@pytest.mark.parametrize("bad", [torch.zeros(128, 11), torch.zeros(128, 10, dtype=torch.int64)])
def test_bad_prompts_raise(bad):
    with pytest.raises(ValueError):
        mixed.plan_row_reuse([bad], 64, 768, (576,))


@pytest.mark.parametrize("compact", [0, 575, 832])
def test_bad_buckets_raise(compact):
    with pytest.raises(ValueError):
        mixed.plan_row_reuse([prompt(128)] * 4, 64, 768, (compact,))


def test_packed_row_slots():
    slots = mixed.packed_row_slots([7, 8, 9], [4, 3], [1, 2, 99], 10)
    assert slots.tolist() == [7, 8, 9, 1, 1, 1, 1, 2, 2, 2, 99, 99, 99]
    with pytest.raises(ValueError):
        mixed.packed_row_slots([0], [4, 3], [1, 2], 10)
    with pytest.raises(ValueError):
        mixed.packed_row_slots([0], [8, 3], [1, 2, 3], 10)


def test_oracle_padding_route_uses_row_zero():
    rng = np.random.default_rng(5)
    logits = O.bf16_round(rng.standard_normal((6, 128)).astype(np.float32))
    slots = np.array([0, 500, 3, 512, 900, 1])
    w, ids = O.route(logits, 8, row_slots=slots, padding_start=512)
    w0, ids0 = O.route(logits, 8)
    for t in range(6):
        src = 0 if slots[t] >= 512 else t
        assert (ids[t] == ids0[src]).all() and (w[t] == w0[src]).all()
