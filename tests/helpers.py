"""Conversions between the oracle's numpy arrays and device tensors, and the
parity metrics used by the GPU tests."""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as O

# Value tolerance of the north star: max-abs 2e-2 and relative L2 1e-2.
MAX_ABS = 2e-2
REL_L2 = 1e-2


def to_bf16(a: np.ndarray, device="cuda") -> torch.Tensor:
    bits = O.bf16_to_bits(np.asarray(a, dtype=np.float32))
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def from_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def to_fp8(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8)).view(torch.float8_e4m3fn).to(device)


def fp8_bytes(t: torch.Tensor) -> np.ndarray:
    return t.detach().view(torch.uint8).cpu().numpy()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.sqrt(((a - b) ** 2).sum() / max((b ** 2).sum(), 1e-30)))


def assert_close(actual, expected, max_abs=MAX_ABS, rel=REL_L2, what=""):
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert np.isfinite(actual).all(), f"{what}: non-finite output"
    err = np.abs(actual - expected).max() if actual.size else 0.0
    r = rel_l2(actual, expected)
    assert err <= max_abs and r <= rel, f"{what}: max-abs {err:.3e} (<= {max_abs}), rel-L2 {r:.3e} (<= {rel})"


def ulps_bf16(a, b) -> np.ndarray:
    ia = (np.asarray(a, np.float32).view(np.int32) >> 16).astype(np.int64)
    ib = (np.asarray(b, np.float32).view(np.int32) >> 16).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFF), ib)
    return np.abs(ia - ib)


def experts_to_oracle(ex) -> "O.Experts":
    """Device ExpertWeights -> oracle container of per-expert numpy arrays."""
    w13 = fp8_bytes(ex.w13_weight)
    w2 = fp8_bytes(ex.w2_weight)
    s13 = ex.w13_scale_inv.cpu().numpy()
    s2 = ex.w2_scale_inv.cpu().numpy()
    return O.Experts(w13, s13, w2, s2)


def assert_logits_close(got, ref, what: str):
    """Two roundings to bf16 of the same fp32-accumulated dot products in
    different summation orders: within one bf16 ulp of each other, or, for
    logits near zero where the sum cancels, within the fp32 accumulation noise
    floor (2^-16 of the row's RMS logit)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if not got.size:
        return
    mag = np.maximum(np.abs(got), np.abs(ref))
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(mag, 1e-30))) - 7)
    floor = np.sqrt((ref ** 2).mean(axis=-1, keepdims=True)) * 2.0 ** -16
    excess = np.abs(got - ref) - np.maximum(ulp, floor)
    bad = np.argwhere(excess > 0)
    assert not len(bad), (f"{what}: {len(bad)} logits beyond one bf16 ulp / the noise floor, e.g. "
                          f"{[(tuple(i), float(got[tuple(i)]), float(ref[tuple(i)])) for i in bad[:4]]}")


def device_logits_routing(x: np.ndarray, router, E: int, k: int, bias: np.ndarray | None = None,
                          chunk: int = 1024):
    """Routing parity for a layer call on x (bf16 values as float32).

    From 256 tokens the router projection runs on the tensor cores, whose fp32
    accumulation order is the hardware's own (the reference's bf16 F.linear is
    the same), so the check is in two parts: (1) the device logits, from the
    same kernel the layer runs at this T, lie within one bf16 ulp of the
    oracle's fixed-order logits (or within the fp32 noise floor for logits
    that cancel to near zero, assert_logits_close); (2) the oracle's top-k of
    the DEVICE logits is what the layer must return, bit for bit. Below 256
    tokens the two logits are identical. Returns (device logits, oracle ids,
    oracle weights) as numpy arrays."""
    from d3moe import ops

    bt = None if bias is None else torch.from_numpy(np.asarray(bias, np.float32)).cuda()
    lg_dev = from_bf16(ops.router_logits(to_bf16(x), router, bias=bt))
    rw = from_bf16(router)
    lg_o = np.concatenate([O.router_logits(x[i:i + chunk], rw, bias, nbias=E)
                           for i in range(0, len(x), chunk)])
    assert_logits_close(lg_dev, lg_o, "router logits vs the oracle's")
    w, ids = O.route(lg_dev[:, :E], k)
    return lg_dev, ids, O.bf16_round(w)

