"""Drop-in for src/drama3/experimental_fp8.py: FP8 128x128 block-scaled dense
projections.

register(weight) quantises a bf16 [N,K] weight into e4m3 blocks with fp32
scales (max(amax,1e-8)/448, experimental_fp8.py:10-18) and keeps it in WEIGHTS
keyed by data_ptr (experimental_fp8.py:7,53). linear(x, weight) computes
x . dequant(W)^T with bf16 activations and fp32 accumulation for every batch
size -- the M=1 arithmetic of the reference (_gemv, :21-29). The reference's
M>=2 branch re-quantised activations and was numerically broken by a scale
layout mismatch; the weight-only form here has no such branch.
"""

from __future__ import annotations

from . import ops

WEIGHTS: dict[int, tuple] = {}


def register(weight):
    n, k = weight.shape
    if k % 128:
        raise ValueError("Experimental dense FP8 needs a 128-aligned reduction width")
    quantized, scales = ops.fp8_quantize_weight(weight.contiguous())
    WEIGHTS[weight.data_ptr()] = (weight, quantized, scales)


def register_quantized(weight_key, quantized, scales, n: int | None = None):
    """Register an already block-quantised weight under `weight_key`'s data_ptr."""
    WEIGHTS[weight_key.data_ptr()] = (weight_key, quantized, scales, n)


def linear(x, weight):
    entry = WEIGHTS[weight.data_ptr()]
    _, quantized, scales = entry[:3]
    n = entry[3] if len(entry) > 3 and entry[3] is not None else weight.shape[0]
    return ops.fp8_gemv(x, quantized, scales, n=n)
