"""Pins the CPU oracle to the reference: every oracle function reproduces the
golden vectors that the reference's own Triton kernels produced
(tests/golden/make_golden.py, Triton interpreter)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import moe_oracle as O

H, E, I = 2048, 256, 512


def ulps_bf16(a, b):
    """Distance in bf16 units in the last place (a, b: bf16 values as f32)."""
    ia = (np.asarray(a, np.float32).view(np.int32) >> 16).astype(np.int64)
    ib = (np.asarray(b, np.float32).view(np.int32) >> 16).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFF), ib)
    return np.abs(ia - ib)


@pytest.mark.parametrize("strided", [0, 1])
@pytest.mark.parametrize("mag", [0, 1, 2, 3])
def test_prepare_moe_input_bytes(golden, strided, mag):
    g = golden("prepare_moe_input")
    k = f"s{strided}_m{mag}"
    x = O.bf16_from_bits(g[k + "_x"])
    router = O.bf16_from_bits(g[k + "_router"])
    qv, _, _ = O.prepare_moe_input(x, router, values=True)
    np.testing.assert_array_equal(qv.view(np.uint32), g[k + "_qf32"].view(np.uint32))
    q, s, lg = O.prepare_moe_input(x, router)
    np.testing.assert_array_equal(q, g[k + "_q"])
    np.testing.assert_array_equal(s.view(np.uint32), g[k + "_scales"].view(np.uint32))
    np.testing.assert_array_equal(lg.view(np.uint32), g[k + "_logits"].view(np.uint32))


def test_e4m3_store_rounding_matches_torch_cast():
    """The byte encoding used after the reference's fp32 values: nearest-even
    E4M3 with saturation, equal to torch's float8_e4m3fn cast (and to the GPU's
    cvt.rn.satfinite.e4m3x2.f32) on every value class."""
    import torch

    rng = np.random.default_rng(3)
    pos = O.E4M3_F32[:127]
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 1, 30, 400)]
                       + [pos, -pos, (pos[:-1] + pos[1:]) / 2, -(pos[:-1] + pos[1:]) / 2]).astype(np.float32)
    v = np.clip(v, -448, 448).astype(np.float32)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(O.e4m3_encode(v), ref)


def test_prepare_moe_input_padding_rows(golden):
    g = golden("prepare_moe_input")
    args = (O.bf16_from_bits(g["pad_x"]), O.bf16_from_bits(g["pad_router"]), g["pad_slots"],
            int(g["pad_start"]))
    qv, _, _ = O.prepare_moe_input(*args, values=True)
    np.testing.assert_array_equal(qv, g["pad_qf32"])
    q, s, lg = O.prepare_moe_input(*args)
    np.testing.assert_array_equal(q, g["pad_q"])
    np.testing.assert_array_equal(s, g["pad_scales"])
    np.testing.assert_array_equal(lg, g["pad_logits"])


def test_route_ids_exact_weights_within_one_ulp(golden):
    g = golden("route")
    w, ids = O.route(O.bf16_from_bits(g["logits"]), 8)
    np.testing.assert_array_equal(ids, g["ids"])
    assert ulps_bf16(O.bf16_round(w), O.bf16_from_bits(g["weights"])).max() <= 1


@pytest.mark.parametrize("T", [1, 5, 37])
@pytest.mark.parametrize("bm", [16, 64])
def test_permute_exact(golden, T, bm):
    g = golden("permute")
    k = f"t{T}_bm{bm}"
    counts, starts, total, sorted_ids, expert_ids = O.moe_permute(g[k + "_ids"], 256, bm)
    np.testing.assert_array_equal(counts, g[k + "_counts"])
    np.testing.assert_array_equal(starts, g[k + "_starts"])
    assert total == int(g[k + "_total"])
    np.testing.assert_array_equal(sorted_ids, g[k + "_sorted"])
    np.testing.assert_array_equal(expert_ids, g[k + "_experts"])


@pytest.fixture(scope="module")
def small(golden):
    g = golden("small_batch")
    sel = g["experts"]
    w13 = {}, {}
    up, ups, dn, dns = {}, {}, {}, {}
    for e in sel:
        up[int(e)], ups[int(e)] = O.synth_expert(int(g["wseed_up"]), int(e), 2 * I, H)
        dn[int(e)], dns[int(e)] = O.synth_expert(int(g["wseed_down"]), int(e), H, I)
    return g, up, ups, dn, dns


def test_activation_quant_matches_reference_inputs(small):
    g = small[0]
    q, s = O.quant_act_fp8(O.bf16_from_bits(g["x"]))
    np.testing.assert_array_equal(q, g["xq"])
    np.testing.assert_array_equal(s, g["xs"])


def test_gate_up_matches_reference(small):
    g, up, ups, _, _ = small
    gu = O.expert_gate_up(g["xq"], g["xs"], up, ups, g["ids"])
    ref = O.bf16_from_bits(g["gate_up"])
    d = ulps_bf16(gu, ref)
    assert d.max() <= 1 and (d > 0).mean() < 0.01


def test_silu_mul_matches_reference(small):
    g = small[0]
    out = O.silu_mul(O.bf16_from_bits(g["gate_up"]))
    assert ulps_bf16(out, O.bf16_from_bits(g["silu_mul"])).max() <= 1


def test_down_combine_matches_reference(small):
    g, _, _, dn, dns = small
    w = O.bf16_from_bits(g["weights"])
    y = O.expert_down_combine(g["a"], g["sa"], dn, dns, g["ids"], w)
    ref = O.bf16_from_bits(g["y"])
    d = ulps_bf16(y, ref)
    assert d.max() <= 2 and (d > 0).mean() < 0.02
    ya = O.bf16_from_bits(g["y_atomic"])
    da = ulps_bf16(y, ya)
    assert da.max() <= 2 and (da > 0).mean() < 0.05


def test_combine_experts_matches_reference(golden):
    g = golden("combine")
    out = O.combine_experts(O.bf16_from_bits(g["routed"]), O.bf16_from_bits(g["shared"]),
                            O.bf16_from_bits(g["gate"]))
    assert ulps_bf16(out, O.bf16_from_bits(g["out"])).max() <= 1


def test_dense_fp8_quantize_and_gemv(golden):
    g = golden("dense_fp8")
    w = O.bf16_from_bits(g["w"])
    qv, _ = O.quantize_weight_blocks(w, values=True)
    np.testing.assert_array_equal(qv, g["qf32"])
    q, s = O.quantize_weight_blocks(w)
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(s, g["s"])
    y = O.fp8_gemv(O.bf16_from_bits(g["x"]), q, s, n=w.shape[0])
    assert ulps_bf16(y, O.bf16_from_bits(g["y"])).max() <= 1
    assert ulps_bf16(y, O.bf16_from_bits(g["y_grouped"])).max() <= 1


def test_router_logits_order_is_a_permutation_of_the_dot_product():
    rng = np.random.default_rng(0)
    x = O.bf16_round(rng.standard_normal((3, 384)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal((5, 384)) * 0.02).astype(np.float32))
    got = O.router_logits(x, w)
    ref = O.bf16_round((x.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float32))
    assert ulps_bf16(got, ref).max() <= 1


def test_add_norm_matches_reference(golden):
    """add_norm (kernels.py:405-423) golden from the reference kernel: the
    residual update and the normalised rows are both bit-exact."""
    g = golden("add_norm")
    out, res = O.add_norm(O.bf16_from_bits(g["x"]), O.bf16_from_bits(g["residual_in"]),
                          O.bf16_from_bits(g["weight"]), float(g["eps"]))
    np.testing.assert_array_equal(O.bf16_to_bits(res), g["residual_out"])
    np.testing.assert_array_equal(O.bf16_to_bits(out), g["out"])


def test_bf16_fma_rounds_once():
    """fma.rn.bf16 semantics of the combine in combine_experts_add_norm
    (kernels.py:464-472): one rounding of the exact a*b + c, which differs from
    rounding the product first (the combine_experts form) on some inputs."""
    rng = np.random.default_rng(3)
    a = O.bf16_round(rng.standard_normal(20000).astype(np.float32))
    b = O.bf16_round(rng.uniform(0, 1, 20000).astype(np.float32))
    c = O.bf16_round(rng.standard_normal(20000).astype(np.float32))
    once = O.bf16_fma(a, b, c)
    exact = a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)
    assert (np.abs(once - exact) <= np.abs(O.bf16_round(exact.astype(np.float32)) - exact) + 0).all()
    twice = O.bf16_round((O.bf16_round((a * b).astype(np.float32)) + c).astype(np.float32))
    assert (once != twice).any()


def test_combine_add_norm_with_zero_shared_is_add_norm(golden):
    """With shared = 0 the fused combine leaves routed unchanged, so
    combine_experts_add_norm reduces to add_norm(routed, residual)."""
    g = golden("add_norm")
    x, res, w = (O.bf16_from_bits(g[k]) for k in ("x", "residual_in", "weight"))
    gate = np.zeros((x.shape[0], 1), np.float32)
    out_c, res_c = O.combine_experts_add_norm(x, np.zeros_like(x), gate, res, w, float(g["eps"]))
    out_a, res_a = O.add_norm(x, res, w, float(g["eps"]))
    np.testing.assert_array_equal(res_c, res_a)
    np.testing.assert_array_equal(out_c, out_a)
