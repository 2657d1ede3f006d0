"""GPU parity of each operator against the pinned oracle and the reference's
golden vectors. All calls go through libd3moe.so (the C ABI)."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import (assert_close, assert_logits_close, fp8_bytes, from_bf16,  # noqa: E402
                     to_bf16, to_fp8, ulps_bf16)
from oracle import moe_oracle as O  # noqa: E402


@pytest.fixture(scope="module")
def d3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from d3moe import experimental_fp8, kernels, moe_input, ops, synth
    return dict(ops=ops, kernels=kernels, moe_input=moe_input, fp8=experimental_fp8, synth=synth)


# ------------------------------------------------------------------- (a3) --
@pytest.mark.parametrize("strided", [0, 1])
@pytest.mark.parametrize("mag", [0, 1, 2, 3])
def test_prepare_moe_input_golden_bytes(d3, golden, strided, mag):
    g = golden("prepare_moe_input")
    k = f"s{strided}_m{mag}"
    x = to_bf16(O.bf16_from_bits(g[k + "_x"]))
    router = to_bf16(O.bf16_from_bits(g[k + "_router"]))
    if strided:  # same values behind the reference's strided views
        xs = torch.zeros((x.shape[0], 4096), dtype=torch.bfloat16, device="cuda")
        xs[:, :2048] = x
        rs = torch.zeros((x.shape[0], 1408), dtype=torch.bfloat16, device="cuda")
        rs[:, :256] = router
        x, router = xs[:, :2048], rs[:, :256]
    q, s, lg = d3["moe_input"].prepare_moe_input(x, router)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(fp8_bytes(q), g[k + "_q"])
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), g[k + "_scales"].view(np.uint32))
    np.testing.assert_array_equal(lg.cpu().numpy().view(np.uint32), g[k + "_logits"].view(np.uint32))


def test_prepare_moe_input_padding_rows(d3, golden):
    g = golden("prepare_moe_input")
    slots = torch.from_numpy(g["pad_slots"]).cuda()
    q, s, lg = d3["moe_input"].prepare_moe_input(
        to_bf16(O.bf16_from_bits(g["pad_x"])), to_bf16(O.bf16_from_bits(g["pad_router"])),
        row_slots=slots, padding_start=int(g["pad_start"]))
    np.testing.assert_array_equal(fp8_bytes(q), g["pad_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), g["pad_scales"])
    np.testing.assert_array_equal(lg.cpu().numpy(), g["pad_logits"])


@pytest.mark.parametrize("T", [1, 7, 64, 300])
def test_quant_act_matches_oracle_bytes(d3, T):
    rng = np.random.default_rng(T)
    x = O.bf16_round((rng.standard_normal((T, 2048)) * rng.choice([1e-3, 1, 50], size=(T, 1))).astype(np.float32))
    x[0, :128] = 0.0  # an all-zero group
    q, s = d3["ops"].quant_act_fp8(to_bf16(x))
    qo, so = O.quant_act_fp8(x)
    np.testing.assert_array_equal(fp8_bytes(q), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


# ------------------------------------------------------------------- (a1) --
# Below 256 tokens the CUDA-core kernel sums in the oracle's fixed order (bit
# for bit); 129/33 rows leave ragged tiles and H=384 a half-filled last
# 256-wide block.
@pytest.mark.parametrize("T,R,H", [(1, 129, 2048), (64, 129, 2048), (13, 257, 2048), (5, 33, 384),
                                   (255, 129, 2048)])
def test_router_logits_bit_exact(d3, T, R, H):
    rng = np.random.default_rng(R + T)
    x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal((R, H)) * 0.02).astype(np.float32))
    got = from_bf16(d3["ops"].router_logits(to_bf16(x), to_bf16(w)))
    np.testing.assert_array_equal(got, O.router_logits(x, w))


def test_router_logits_gathered_rows_match_materialised_rows(d3):
    """A layer call through a keep map (rows gathered in the library) routes
    exactly like the call on the materialised rows x[keep] (the reference's
    index_select), on both router paths (kept rows below and from 256)."""
    from d3moe import synth
    lw = synth.make_layer(128, 768, 2048, seed=4, device="cuda")
    rng = np.random.default_rng(12)
    x = to_bf16(O.bf16_round(rng.standard_normal((340, 2048)).astype(np.float32)))
    for n in (200, 300):
        keep = torch.from_numpy(np.sort(rng.choice(340, n, replace=False)).astype(np.int64)).cuda()
        out_k, ids_k, w_k = d3["ops"].moe_layer(x, lw.router, lw.experts, lw.shared, 8, keep=keep,
                                                return_routing=True)
        out_m, ids_m, w_m = d3["ops"].moe_layer(x.index_select(0, keep), lw.router, lw.experts, lw.shared,
                                                8, return_routing=True)
        torch.cuda.synchronize()
        assert torch.equal(ids_k, ids_m) and torch.equal(w_k, w_m), n
        assert torch.equal(out_k, out_m), n


def _router_exact(x, w, bias=None):
    """float64 value of x . w^T (+ bias) before the bf16 rounding."""
    v = x.astype(np.float64) @ w.astype(np.float64).T
    if bias is not None:
        v[:, : len(bias)] += bias
    return v


# From 256 tokens the projection is a tcgen05 bf16 GEMM (fp32 accumulation in
# the tensor core's order): every logit is the float64 value rounded to bf16 up
# to fp32 accumulation noise, within one bf16 ulp (or the noise floor) of the
# oracle, and bit-identical from call to call. 300 tokens and 129/33 rows
# leave ragged tiles; 257 rows take two 144-row tiles; H=384 and 4096 change
# the K loop; a bias on the first R-1 columns is added before the rounding.
@pytest.mark.parametrize("T,R,H,biased", [(256, 129, 2048, False), (300, 129, 2048, True),
                                          (513, 33, 384, False), (260, 17, 4096, False),
                                          (300, 257, 2048, True), (4100, 129, 2048, True)])
def test_router_logits_tensor_core(d3, T, R, H, biased):
    rng = np.random.default_rng(R + T + H)
    x = O.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    w = O.bf16_round((rng.standard_normal((R, H)) * 0.02).astype(np.float32))
    bias = rng.standard_normal(R - 1).astype(np.float32) if biased else None
    bt = None if bias is None else torch.from_numpy(bias).cuda()
    got = d3["ops"].router_logits(to_bf16(x), to_bf16(w), bias=bt)
    again = d3["ops"].router_logits(to_bf16(x), to_bf16(w), bias=bt)
    torch.cuda.synchronize()
    assert torch.equal(got, again)
    g = from_bf16(got)
    exact = _router_exact(x, w, bias)
    # the float64 value rounded once to bf16, up to fp32 accumulation noise
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 1e-30))) - 7)
    noise = np.sqrt((exact ** 2).mean(axis=1, keepdims=True)) * 2.0 ** -16
    excess = np.abs(g - exact) - (0.5 * ulp + noise)
    bad = np.argwhere(excess > 0)
    assert not len(bad), (f"{len(bad)} logits above the rounding bound, e.g. "
                          f"{[(tuple(i), float(g[tuple(i)]), float(exact[tuple(i)])) for i in bad[:4]]}")
    s = slice(0, min(T, 600))
    assert_logits_close(g[s], O.router_logits(x[s], w, bias, nbias=None if bias is None else R - 1),
                        "tensor-core router vs the oracle")


# ------------------------------------------------------------------- (a2) --
def test_route_golden(d3, golden):
    g = golden("route")
    w, ids = d3["kernels"].route(to_bf16(O.bf16_from_bits(g["logits"])))
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])
    assert ulps_bf16(from_bf16(w), O.bf16_from_bits(g["weights"])).max() <= 1


@pytest.mark.parametrize("E", [128, 256, 1000])
def test_route_matches_oracle(d3, E):
    rng = np.random.default_rng(E)
    lg = O.bf16_round(rng.standard_normal((97, E)).astype(np.float32))
    lg[3, :] = lg[3, 0]           # an all-equal row: ids 0..7
    lg[4, 17] = lg[4, 3] = 9.0    # a tie at the top
    bias = rng.standard_normal(E).astype(np.float32)
    w, ids = d3["ops"].route_topk(to_bf16(lg), 8)
    wo, io = O.route(lg, 8)
    np.testing.assert_array_equal(ids.cpu().numpy(), io)
    assert ulps_bf16(from_bf16(w), O.bf16_round(wo)).max() <= 1
    wb, ib = d3["ops"].route_topk(to_bf16(lg), 8, bias=torch.from_numpy(bias).cuda(),
                                  weights_dtype=torch.float32)
    wob, iob = O.route(lg, 8, bias=bias)
    np.testing.assert_array_equal(ib.cpu().numpy(), iob)
    np.testing.assert_allclose(wb.cpu().numpy(), wob, rtol=1e-5, atol=1e-7)


# ------------------------------------------------------------------- (a4) --
@pytest.mark.parametrize("T", [1, 5, 37])
@pytest.mark.parametrize("bm", [16, 64])
def test_permute_golden(d3, golden, T, bm):
    g = golden("permute")
    k = f"t{T}_bm{bm}"
    ids = torch.from_numpy(g[k + "_ids"]).cuda()
    counts, starts, total, sorted_ids, expert_ids = d3["kernels"].moe_permute(ids, 256, bm)
    tot = int(g[k + "_total"])
    assert int(total.item()) == tot
    np.testing.assert_array_equal(counts.cpu().numpy(), g[k + "_counts"])
    np.testing.assert_array_equal(starts.cpu().numpy(), g[k + "_starts"])
    np.testing.assert_array_equal(sorted_ids.cpu().numpy()[:tot], g[k + "_sorted"])
    np.testing.assert_array_equal(expert_ids.cpu().numpy()[: tot // bm], g[k + "_experts"])
    assert (sorted_ids.cpu().numpy()[tot:] == T * 8).all()


@pytest.mark.parametrize("chunked", [False, True])
@pytest.mark.parametrize("T,E,bm", [(64, 128, 1), (2048, 128, 64), (8192, 128, 128), (3, 1000, 16),
                                    (8192, 128, 1), (40000, 1000, 1)])
def test_permute_matches_oracle(d3, T, E, bm, chunked):
    """chunked=True: three multi-CTA kernels from 8192 pairs (below that the
    entry falls back to the one-CTA kernel); outputs must be identical."""
    rng = np.random.default_rng(T + E)
    hot = rng.zipf(1.5, size=(T, 8)) % E  # skewed, with duplicate experts across tokens
    ids = np.stack([rng.permutation(E)[:8] if t % 3 else (hot[t] + np.arange(8)) % E for t in range(T)])
    ids = ids.astype(np.int64)
    counts, starts, total, sorted_ids, expert_ids, inv, active, n_active = d3["ops"].moe_permute(
        torch.from_numpy(ids).cuda(), E, bm, chunked=chunked)
    c, s, tot, so, eo = O.moe_permute(ids, E, bm)
    assert int(total.item()) == tot
    np.testing.assert_array_equal(counts.cpu().numpy(), c)
    np.testing.assert_array_equal(starts.cpu().numpy(), s)
    np.testing.assert_array_equal(sorted_ids.cpu().numpy()[:tot], so)
    np.testing.assert_array_equal(expert_ids.cpu().numpy()[: tot // bm], eo)
    invn = inv.cpu().numpy()
    np.testing.assert_array_equal(sorted_ids.cpu().numpy()[invn], np.arange(T * 8))
    na = int(n_active.item())
    np.testing.assert_array_equal(active.cpu().numpy()[:na], np.nonzero(c)[0])


# ------------------------------------------------------------------- (a6) --
def test_silu_mul_golden(d3, golden):
    g = golden("small_batch")
    out = d3["kernels"].silu_mul(to_bf16(O.bf16_from_bits(g["gate_up"])))
    assert ulps_bf16(from_bf16(out), O.bf16_from_bits(g["silu_mul"])).max() <= 1


def test_silu_mul_quant_matches_oracle(d3):
    rng = np.random.default_rng(5)
    gu = O.bf16_round(rng.standard_normal((37, 1536)).astype(np.float32))
    q, s = d3["ops"].silu_mul_quant(to_bf16(gu))
    qo, so = O.silu_mul_quant(gu)
    # sigmoid may differ in the last fp32 bit from numpy's exp: allow rare 1-code flips
    qb = fp8_bytes(q)
    assert (qb != qo).mean() < 1e-3
    np.testing.assert_allclose(s.cpu().numpy(), so, rtol=1e-6)


# ------------------------------------------------------------------- (a9) --
def test_combine_experts_golden(d3, golden):
    g = golden("combine")
    out = d3["kernels"].combine_experts(to_bf16(O.bf16_from_bits(g["routed"])),
                                        to_bf16(O.bf16_from_bits(g["shared"])),
                                        to_bf16(O.bf16_from_bits(g["gate"])))
    assert ulps_bf16(from_bf16(out), O.bf16_from_bits(g["out"])).max() <= 1


# ------------------------------------------------------------------ (a10) --
def test_dense_fp8_golden(d3, golden):
    g = golden("dense_fp8")
    w = to_bf16(O.bf16_from_bits(g["w"]))
    d3["fp8"].register(w)
    _, q, s = d3["fp8"].WEIGHTS[w.data_ptr()]
    np.testing.assert_array_equal(fp8_bytes(q), g["q"])
    np.testing.assert_array_equal(s.cpu().numpy(), g["s"])
    y = d3["fp8"].linear(to_bf16(O.bf16_from_bits(g["x"])), w)
    assert ulps_bf16(from_bf16(y), O.bf16_from_bits(g["y"])).max() <= 1


@pytest.mark.parametrize("T", [1, 64])
def test_dense_fp8_gemv_every_e4m3_code(d3, T):
    """Weights holding every non-NaN E4M3 code (zeros, subnormals, +-448) in
    every position of a 128-byte row, and activations spanning many binades
    within a group (so the activation split meets tiny elements): the result
    is the float64 value correctly rounded, up to fp32 summation-order noise."""
    codes = np.array([c for c in range(256) if c not in (0x7F, 0xFF)], np.uint8)
    N, K = 256, 512
    idx = (np.arange(N)[:, None] * 7 + np.arange(K)[None, :]) % len(codes)
    q = codes[idx]
    rng = np.random.default_rng(11)
    s = rng.uniform(1e-4, 1e-2, (N // 128, K // 128)).astype(np.float32)
    x = O.bf16_round((rng.standard_normal((T, K)) * np.exp(rng.uniform(-12, 3, (T, K)))).astype(np.float32))
    y = d3["ops"].fp8_gemv(to_bf16(x), to_fp8(q), torch.from_numpy(s).cuda(), n=N)
    got = from_bf16(y)
    exact = x.astype(np.float64) @ O.dequant_blocks(q, s).astype(np.float64).T
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 1e-30))) - 7)
    bound = 0.5 * ulp + np.sqrt((exact ** 2).mean()) * 2.0 ** -16
    assert (np.abs(got - exact) <= bound).all()


@pytest.mark.parametrize("T", [1, 8, 16, 32, 64, 100])
# the benchmark's QKV and o_proj, an odd size, and the reference model's real
# projections: QKV 9216x2048, GDN in 12352x2048, out / o_proj 2048x4096
# (src/drama3/model.py:210-225)
@pytest.mark.parametrize("N,K", [(4096, 2048), (2048, 2048), (300, 384), (9216, 2048), (12352, 2048),
                                 (2048, 4096)])
def test_dense_fp8_gemv_matches_oracle(d3, T, N, K):
    rng = np.random.default_rng(T * 7 + N)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    q, s = O.quantize_weight_blocks(w)
    x = O.bf16_round(rng.standard_normal((T, K)).astype(np.float32))
    y = d3["ops"].fp8_gemv(to_bf16(x), to_fp8(q), torch.from_numpy(s).cuda(), n=N)
    ref = O.fp8_gemv(x, q, s, n=N)
    got = from_bf16(y)
    # Exact value of the same dequantise-then-matmul in float64: the kernel must
    # return it correctly rounded to bf16, up to fp32 summation-order noise
    # (half a bf16 ulp + 2^-16 of the output rms).
    exact = x.astype(np.float64) @ O.dequant_blocks(q, s)[:N].astype(np.float64).T
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 1e-30))) - 7)
    bound = 0.5 * ulp + np.sqrt((exact ** 2).mean()) * 2.0 ** -16
    excess = np.abs(got - exact) - bound
    assert (excess <= 0).all(), float(excess.max())
    assert_close(got, ref, what="dense gemv")


# ---------------------------------------------------------------- (a5-a7) --
def test_small_batch_moe_golden(d3, golden):
    """Drama-3 geometry (E=256, I=512): routed output vs the reference's
    expert_up -> silu_mul_quant -> expert_down chain."""
    g = golden("small_batch")
    E, I, H = 256, 512, 2048
    sel = [int(e) for e in g["experts"]]
    w13 = np.zeros((E, 2 * I, H), np.uint8)
    s13 = np.ones((E, 2 * I // 128, H // 128), np.float32)
    w2 = np.zeros((E, H, I), np.uint8)
    s2 = np.ones((E, H // 128, I // 128), np.float32)
    for e in sel:
        w13[e], s13[e] = O.synth_expert(int(g["wseed_up"]), e, 2 * I, H)
        w2[e], s2[e] = O.synth_expert(int(g["wseed_down"]), e, H, I)
    ex = d3["synth"].ExpertWeights(to_fp8(w13), torch.from_numpy(s13).cuda(), to_fp8(w2),
                                   torch.from_numpy(s2).cuda())
    x = to_bf16(O.bf16_from_bits(g["x"]))
    ids = torch.from_numpy(g["ids"]).cuda()
    w = to_bf16(O.bf16_from_bits(g["weights"]))
    y = d3["kernels"].small_batch_moe(x, ids, w, ex)
    ref = O.bf16_from_bits(g["y"])
    assert_close(from_bf16(y), ref, what="small_batch_moe vs reference")
    y2 = d3["kernels"].native_moe(x, ids, w, ex)
    np.testing.assert_array_equal(from_bf16(y2), from_bf16(y))
