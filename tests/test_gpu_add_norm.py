"""GPU parity of the layer exit (residual update + Gemma RMSNorm), standalone
and fused into the MoE layer's final kernel. Given the same combine inputs the
residual update involves no reduction, so it is bit-exact against the oracle;
the normalised rows differ from the oracle only through the fp32
sum-of-squares order and rsqrt, so they are held to one bf16 ulp. Through the
whole layer the MoE output's own tolerance carries over."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import device_logits_routing, experts_to_oracle, from_bf16, rel_l2, to_bf16, ulps_bf16  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402


@pytest.fixture(scope="module")
def d3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import kernels, ops
    return {"ops": ops, "kernels": kernels}


def _bits(t):
    return O.bf16_to_bits(from_bf16(t))


def test_add_norm_golden(d3, golden):
    g = golden("add_norm")
    x = to_bf16(O.bf16_from_bits(g["x"]))
    res = to_bf16(O.bf16_from_bits(g["residual_in"]))
    w = to_bf16(O.bf16_from_bits(g["weight"]))
    out = d3["kernels"].add_norm(x, res, w, float(g["eps"]))
    np.testing.assert_array_equal(_bits(res), g["residual_out"])
    assert ulps_bf16(from_bf16(out), O.bf16_from_bits(g["out"])).max() <= 1


@pytest.mark.parametrize("W", [2048, 4096, 1000])
def test_combine_experts_add_norm_matches_oracle(d3, W):
    rng = np.random.default_rng(W)
    T = 37
    routed = O.bf16_round((rng.standard_normal((T, W)) * 0.3).astype(np.float32))
    shared = O.bf16_round((rng.standard_normal((T, W)) * 0.3).astype(np.float32))
    packed = O.bf16_round((rng.standard_normal((T, 17)) * 2.0).astype(np.float32))  # gate column 5, stride 17
    res = O.bf16_round((rng.standard_normal((T, W)) * 2.0).astype(np.float32))
    w = O.bf16_round((rng.standard_normal(W) * 0.1).astype(np.float32))
    pt = to_bf16(packed)
    gate = pt[:, 5:6]
    rt = to_bf16(res)
    out = d3["kernels"].combine_experts_add_norm(to_bf16(routed), to_bf16(shared), gate, rt, to_bf16(w), 1e-6)
    out_o, res_o = O.combine_experts_add_norm(routed, shared, packed[:, 5:6], res, w, 1e-6)
    np.testing.assert_array_equal(_bits(rt), O.bf16_to_bits(res_o))
    assert ulps_bf16(from_bf16(out), out_o).max() <= 1


def test_combine_experts_add_norm_inverse(d3):
    """Compact routed/shared rows gathered by an inverse map (kernels.py:502-556):
    several residual rows may read the same source row."""
    rng = np.random.default_rng(9)
    T, S, W = 29, 11, 2048
    routed = O.bf16_round((rng.standard_normal((S, W)) * 0.3).astype(np.float32))
    shared = O.bf16_round((rng.standard_normal((S, W)) * 0.3).astype(np.float32))
    gate = O.bf16_round(rng.standard_normal((S, 1)).astype(np.float32))
    inverse = rng.integers(0, S, size=T)
    res = O.bf16_round(rng.standard_normal((T, W)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal(W) * 0.1).astype(np.float32))
    rt = to_bf16(res)
    out = d3["kernels"].combine_experts_add_norm_inverse(
        to_bf16(routed), to_bf16(shared), to_bf16(gate), torch.from_numpy(inverse).cuda(), rt,
        to_bf16(w), 1e-6)
    out_o, res_o = O.combine_experts_add_norm(routed, shared, gate, res, w, 1e-6, inverse=inverse)
    np.testing.assert_array_equal(_bits(rt), O.bf16_to_bits(res_o))
    assert ulps_bf16(from_bf16(out), out_o).max() <= 1


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import synth
    E, I, H = 128, 768, 2048
    lw = synth.make_layer(E, I, H, seed=21, device="cuda")
    return lw, experts_to_oracle(lw.experts), experts_to_oracle(lw.shared)


@pytest.mark.parametrize("T,prefill", [(16, False), (64, False), (300, True)])
def test_fused_layer_exit_matches_two_step(d3, layer, T, prefill):
    """moe_layer(..., residual, norm_weight) equals moe_parts followed by
    combine_experts_add_norm bit for bit (same routed/shared rounding, same
    norm kernel), and matches the oracle within the layer tolerance."""
    from d3moe.model import MoE
    ops = d3["ops"]
    lw, ex, sh = layer
    H = 2048
    rng = np.random.default_rng(T)
    x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    res0 = O.bf16_round((rng.standard_normal((T, H)) * 2.0).astype(np.float32))
    nw = O.bf16_round((rng.standard_normal(H) * 0.1).astype(np.float32))
    xt, nwt = to_bf16(x), to_bf16(nw)
    threshold = 1 if prefill else 1 << 30
    with ops.prefill_min_tokens(threshold):
        r_fused = to_bf16(res0)
        out_fused = ops.moe_layer(xt, lw.router, lw.experts, lw.shared, 8, residual=r_fused, norm_weight=nwt)

        class L:
            experts = lw.experts
            shared_expert = lw.shared
            router_weight = lw.router

        routed, shared, gate = MoE().moe_parts(xt, L)
        r_two = to_bf16(res0)
        out_two = d3["kernels"].combine_experts_add_norm(routed, shared, gate, r_two, nwt, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(r_fused, r_two)
    assert torch.equal(out_fused, out_two)
    logits, ids_o, w_o = device_logits_routing(x, lw.router, 128, 8)
    routed_o, sh_o = O.moe_experts(x, ids_o, w_o, ex, sh, rows_bf16=prefill)
    out_o, res_o = O.combine_experts_add_norm(routed_o, sh_o, logits[:, 128:129], res0, nw, 1e-6)
    # the residual (|v| up to ~8) and the normalised rows carry the MoE output's
    # tolerance-level differences (max-abs 2e-2) through one more bf16 rounding
    # of values above 1 (one ulp of the value); relative L2 stays at 1e-2
    def within(actual, expected, what):
        a = np.asarray(actual, np.float64)
        ulp = np.spacing(np.abs(expected).astype(np.float32)).astype(np.float64) * 65536.0
        assert (np.abs(a - expected) <= 2e-2 + ulp).all(), what
        assert rel_l2(a, expected) <= 1e-2, what

    rf = from_bf16(r_fused).astype(np.float64)
    within(rf, res_o, f"fused exit residual T={T}")
    assert rel_l2(rf - res0, res_o - res0) <= 1e-2, f"fused exit residual update T={T}"
    within(from_bf16(out_fused), out_o, f"fused exit out T={T}")
