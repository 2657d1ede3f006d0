"""Gated single-request projection with the reference's signature
(src/drama3/fused_projection.py:39-60) on FP8 weights.

The weight is the bf16 projection weight registered with
`d3moe.experimental_fp8.register` (which keeps its 128x128 block-quantised
FP8 copy); the gate is applied in the GEMV's activation prep:
activated = bf16(x * bf16(silu(gate))) ("swiglu") or bf16(x * bf16(sigmoid(gate)))
("sigmoid"), then y = activated . dequant(Wq, S)^T with fp32 accumulation.
`rows` and `warps` (Triton tile knobs) are accepted and ignored."""

from __future__ import annotations

import torch

from . import experimental_fp8, ops


def gated_gemv(x, gate, weight, mode, rows=None, warps=None):
    if x.shape[0] != 1 or x.dtype != torch.bfloat16:
        raise ValueError("Fused gating requires one BF16 row")
    if mode not in ("swiglu", "sigmoid"):
        raise ValueError("Expected swiglu or sigmoid")
    entry = experimental_fp8.WEIGHTS.get(weight.data_ptr())
    if entry is None:
        raise KeyError("gated_gemv needs the weight registered with d3moe.experimental_fp8.register")
    _, quantized, scales = entry[:3]
    n = entry[3] if len(entry) > 3 and entry[3] is not None else weight.shape[0]
    return ops.fp8_gated_gemv(x, gate.reshape(1, -1), quantized, scales, mode, n=n)
