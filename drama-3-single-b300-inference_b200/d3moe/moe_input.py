"""Drop-in for src/drama3/moe_input.py: fused activation FP8 quantisation and
router-logit conversion (prepare_moe_input, moe_input.py:40-79)."""

from __future__ import annotations

import torch

from . import ops
from ._lib import call


def prepare_moe_input(x, router, *, row_slots=None, padding_start=None):
    """Returns (q e4m3 [T,H], scales f32 [H/128, T], logits f32 [T,E]).

    Optionally reuse row 0 routing for reserved padding slots (rows whose slot
    is >= padding_start), exactly as the reference. Raises ValueError on the
    reference's shape/stride/flag errors (moe_input.py:47-62)."""
    if x.dim() != 2 or router.dim() != 2 or router.shape[0] != x.shape[0]:
        raise ValueError("Expected hidden [T,H] and router [T,E] with matching rows")
    if x.shape[1] % 128:
        raise ValueError("Expected a hidden size that is a multiple of 128")
    if x.stride(1) != 1 or router.stride(1) != 1:
        raise ValueError("Channel strides must be contiguous")
    if (row_slots is None) != (padding_start is None):
        raise ValueError("Reserved padding routing requires both row_slots and padding_start")
    if row_slots is not None:
        if (
            row_slots.shape != (len(x),)
            or row_slots.stride(0) != 1
            or row_slots.device != x.device
            or row_slots.dtype not in (torch.int32, torch.int64)
        ):
            raise ValueError("Expected one contiguous integer slot per MoE row on the same device")
        if not isinstance(padding_start, int) or padding_start <= 0:
            raise ValueError("padding_start must be a positive reserved-slot boundary")
    ops._require_cuda(x, router, row_slots)
    T, H = x.shape
    E = router.shape[1]
    q = torch.empty(x.shape, device=x.device, dtype=torch.float8_e4m3fn)
    scales = torch.empty((H // 128, T), device=x.device, dtype=torch.float32)
    logits = torch.empty((T, E), device=x.device, dtype=torch.float32)
    call("d3_prepare_moe_input", x.data_ptr(), x.stride(0), router.data_ptr(), router.stride(0),
         T, H, E, None if row_slots is None else row_slots.data_ptr(),
         int(row_slots is not None and row_slots.dtype == torch.int64), padding_start or 0,
         q.data_ptr(), scales.data_ptr(), logits.data_ptr(), ops._stream(x.device))
    return q, scales, logits
