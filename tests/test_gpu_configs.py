"""GPU parity at the benchmark configurations themselves, with their stated
seeds and sizes (H=2048, E=128, I=768, top-8, N(0, 0.02) weights quantised
per 128x128 block, bf16 N(0, 1) inputs):

  config 1  one decode token, seed 0, the whole layer against the oracle;
  config 2  decode batches 1, 8, 16, 32, 64 at seed 1, with the FP8 QKV
            [2048 -> 4096] and o_proj [2048 -> 2048] projections in front of
            the layer, each stage against the oracle;
  config 4  the ragged prefill batch (64 prompts uniform in [16, 512], seed 3,
            Zipf(1.1) router bias) on the tcgen05 path;
  8192      the prefill target size (seed 4) on the tcgen05 path.

At prefill sizes the oracle's expert arithmetic is too slow for every token,
so those checks take two parts: the routing ids of EVERY token, bit-exact
against the oracle's router projection and top-k, and the output values of
256 randomly sampled tokens, recomputed by the oracle from those tokens'
routing (a token's output depends on its own routing only; the combine sums
its k expert rows in a fixed order). Values: max-abs 2e-2, rel-L2 1e-2."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from helpers import assert_close, device_logits_routing, experts_to_oracle, from_bf16, to_bf16, ulps_bf16  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

E, I, H, K = 128, 768, 2048, 8
N_QKV, N_O = 4096, 2048
SAMPLED = 256


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _x(T: int, seed: int) -> np.ndarray:
    """bf16 N(0,1) activations from a seeded CPU generator (as float32)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return torch.randn((T, H), generator=g).to(torch.bfloat16).float().numpy()


def _layer(seed: int, router_bias=None):
    from d3moe import synth
    lw = synth.make_layer(E, I, H, seed=seed, device="cuda", router_bias=router_bias)
    return lw, experts_to_oracle(lw.experts), experts_to_oracle(lw.shared)




def _check_prefill(lw, ex, sh, x: np.ndarray, bias: np.ndarray | None, seed: int, what: str):
    from d3moe import ops
    T = len(x)
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    bt = None if bias is None else torch.from_numpy(bias).cuda()
    # the library's default token threshold (1024) puts these sizes on the
    # tcgen05 kernels; it is set explicitly so an environment override cannot
    # move them to the decode engine
    assert T >= 1024
    with ops.prefill_min_tokens(1024):
        out, ids, w = ops.moe_layer(to_bf16(x), lw.router, lw.experts, lw.shared, K, router_bias=bt,
                                    return_routing=True, status=status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    logits, ids_o, w_o = device_logits_routing(x, lw.router, E, K, bias=bias)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o, err_msg=f"{what}: routing ids")
    assert ulps_bf16(from_bf16(w), w_o).max() <= 1, f"{what}: routing weights"
    rng = np.random.default_rng(seed)
    s = np.sort(rng.choice(T, size=min(SAMPLED, T), replace=False))
    routed, shared = O.moe_experts(x[s], ids_o[s], w_o[s], ex, sh, rows_bf16=True)
    ref = O.combine_experts(routed, shared, logits[s, E])
    assert_close(from_bf16(out)[s], ref, what=f"{what}: {len(s)} sampled tokens")


def test_config1_single_decode_token_seed0():
    """Config 1 as written: T=1, seed 0, decode path, whole layer."""
    _need_cuda()
    from d3moe import ops
    lw, ex, sh = _layer(0)
    x = _x(1, 0)
    out, ids, w = ops.moe_layer(to_bf16(x), lw.router, lw.experts, lw.shared, K, return_routing=True)
    ref, ids_o, w_o = O.moe_layer(x, from_bf16(lw.router), ex, sh, K)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    assert ulps_bf16(from_bf16(w), w_o).max() <= 1
    assert_close(from_bf16(out), ref, what="config 1")


def _check_gemv(got, x, q, s, what):
    """The dense GEMV must return the float64 value of the same
    dequantise-then-matmul correctly rounded to bf16, up to fp32
    summation-order noise (half a bf16 ulp + 2^-16 of the output rms), and
    match the oracle within the layer tolerance."""
    exact = x.astype(np.float64) @ O.dequant_blocks(q, s).astype(np.float64).T
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 1e-30))) - 7)
    bound = 0.5 * ulp + np.sqrt((exact ** 2).mean()) * 2.0 ** -16
    excess = np.abs(got - exact) - bound
    assert (excess <= 0).all(), f"{what}: {float(excess.max())} above the rounding bound"
    assert_close(got, O.fp8_gemv(x, q, s), what=what)


@pytest.fixture(scope="module")
def config2():
    _need_cuda()
    from d3moe import synth
    lw, ex, sh = _layer(1)
    g = torch.Generator(device="cpu")
    g.manual_seed(1)
    dense = []
    for n in (N_QKV, N_O):
        wq, s = synth.block_quantize(torch.randn((n, H), generator=g) * 0.02)
        dense.append((wq.cuda(), s.cuda(), wq.view(torch.uint8).numpy(), s.numpy()))
    return lw, ex, sh, dense, _x(64, 1)


@pytest.mark.parametrize("T", [1, 8, 16, 32, 64])
def test_config2_decode_step_seed1(config2, T):
    """Config 2: QKV GEMV -> o_proj GEMV (on the first 2048 QKV columns) ->
    MoE layer, at seed 1. Each stage is checked against the oracle applied to
    the device's own input of that stage, so a last-bit difference upstream
    cannot move the routing of the stage under test."""
    from d3moe import ops
    lw, ex, sh, dense, x64 = config2
    (wq, sq, wq_np, sq_np), (wo, so, wo_np, so_np) = dense
    x = x64[:T]
    qkv = ops.fp8_gemv(to_bf16(x), wq, sq)
    o = ops.fp8_gemv(qkv[:, :H], wo, so)
    out, ids, w = ops.moe_layer(o, lw.router, lw.experts, lw.shared, K, return_routing=True)
    qkv_h, o_h = from_bf16(qkv), from_bf16(o)
    _check_gemv(qkv_h, x, wq_np, sq_np, "QKV")
    _check_gemv(o_h, qkv_h[:, :H], wo_np, so_np, "o_proj")
    ref, ids_o, w_o = O.moe_layer(o_h, from_bf16(lw.router), ex, sh, K)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_o)
    assert ulps_bf16(from_bf16(w), w_o).max() <= 1
    assert_close(from_bf16(out), ref, what=f"config 2 T={T}")


def test_config4_ragged_prefill_zipf_bias():
    """Config 4: 64 prompts with lengths uniform in [16, 512] (seed 3), all
    tokens in one layer call, Zipf(1.1) router bias (hot experts)."""
    _need_cuda()
    lens = np.random.default_rng(3).integers(16, 513, size=64)
    T = int(lens.sum())
    lw, ex, sh = _layer(3, router_bias="zipf")
    bias = lw.router_bias.float().cpu().numpy()
    _check_prefill(lw, ex, sh, _x(T, 3), bias, seed=3, what=f"config 4 T={T}")


def test_prefill_8192_tokens_seed4():
    """The 8192-token prefill target (config 5's prefill batch size), seed 4."""
    _need_cuda()
    lw, ex, sh = _layer(4)
    _check_prefill(lw, ex, sh, _x(8192, 4), None, seed=4, what="prefill T=8192")
