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
