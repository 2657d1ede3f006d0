"""Tensor-level wrappers over the C ABI (include/d3moe.h).

Each wrapper validates dtypes/devices the way the reference's operators do,
allocates its outputs (and workspace) with torch.empty on the input's device
-- the graph pool during CUDA-graph capture -- and enqueues the kernels on the
current torch stream. Nothing here synchronises, so every call can be
captured in a CUDA graph like the reference's decode step
(src/drama3/engine.py:84-92).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import D3Experts, D3Rows, call

FP8 = torch.float8_e4m3fn


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("d3moe operators take CUDA tensors; there is no CPU path")


def _row_stride(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("Channel strides must be contiguous")
    return t.stride(0)


class ExpertView:
    """Read-only view of an expert container as a d3_experts_t.

    `experts` is any object exposing w13_weight [E,2I,H] e4m3, w13_scale_inv
    [E,2I/128,H/128] f32, w2_weight [E,H,I] e4m3 and w2_scale_inv
    [E,H/128,I/128] f32 (the reference's container, src/drama3/kernels.py:
    336-350). gate_up_order: "gate_up" (w13 rows [gate | up], the checkpoint
    order) or "up_gate" ([up | gate], FlashInfer's order, model.py:196-201). `tensors`
    = (w13, s13, w2, s2) replaces the container."""

    def __init__(self, experts=None, gate_up_order: str = "gate_up", *, tensors=None):
        if tensors is not None:
            w13, s13, w2, s2 = tensors
        else:
            w13, s13 = experts.w13_weight, experts.w13_scale_inv
            w2, s2 = experts.w2_weight, experts.w2_scale_inv
        if gate_up_order not in ("gate_up", "up_gate"):
            raise ValueError("gate_up_order must be 'gate_up' or 'up_gate'")
        if w13.dim() == 2:  # a single (shared) expert stored without the E axis
            w13, s13, w2, s2 = w13[None], s13[None], w2[None], s2[None]
        E, I2, H = w13.shape
        I = I2 // 2
        if w13.dtype != FP8 or w2.dtype != FP8:
            raise ValueError("expert weights must be float8_e4m3fn")
        if s13.dtype != torch.float32 or s2.dtype != torch.float32:
            raise ValueError("expert scales must be float32")
        if tuple(w2.shape) != (E, H, I):
            raise ValueError(f"w2_weight shape {tuple(w2.shape)} != {(E, H, I)}")
        if tuple(s13.shape) != (E, I2 // 128, H // 128) or tuple(s2.shape) != (E, H // 128, I // 128):
            raise ValueError("scale shapes must be [E, rows/128, cols/128]")
        for t in (w13, s13, w2, s2):
            if not t.is_contiguous():
                raise ValueError("expert tensors must be contiguous")
        _require_cuda(w13, s13, w2, s2)
        self.tensors = (w13, s13, w2, s2)
        self.E, self.I, self.H = E, I, H
        self.gate_up_order = gate_up_order
        self.struct = D3Experts(w13.data_ptr(), s13.data_ptr(), w2.data_ptr(), s2.data_ptr(), E, I, H,
                                _lib.D3_UP_GATE if gate_up_order == "up_gate" else _lib.D3_GATE_UP)


def quant_act_fp8(x: torch.Tensor, transposed: bool = False):
    """x bf16 [T,H] -> (q e4m3 [T,H], scales f32 [T,H/128] or [H/128,T])."""
    _require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("x must be bfloat16")
    T, H = x.shape
    q = torch.empty((T, H), dtype=FP8, device=x.device)
    s = torch.empty((H // 128, T) if transposed else (T, H // 128), dtype=torch.float32, device=x.device)
    call("d3_quant_act_fp8", x.data_ptr(), _row_stride(x), T, H, q.data_ptr(), s.data_ptr(),
         int(transposed), _stream(x.device))
    return q, s


def router_logits(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 logits [T,R] = bf16(x . weight^T + bias) with fp32 accumulation
    (bias f32 on the first len(bias) columns, before the rounding). Below 256
    tokens the sum runs in the oracle's fixed order; from 256 tokens on the
    tensor cores (the kernels d3_moe_layer uses at the same T)."""
    _require_cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("router projection takes bf16 x and weight")
    T, H = x.shape
    R = weight.shape[0]
    if weight.shape[1] != H or not weight.is_contiguous():
        raise ValueError("router weight must be contiguous [R, H]")
    nbias = 0
    if bias is not None:
        _require_cuda(bias)
        if bias.dtype != torch.float32 or bias.dim() != 1 or not bias.is_contiguous() or bias.numel() > R:
            raise ValueError("router bias must be a contiguous float32 vector of at most R entries")
        nbias = bias.numel()
    out = torch.empty((T, R), dtype=torch.bfloat16, device=x.device)
    call("d3_router_logits", x.data_ptr(), _row_stride(x), weight.data_ptr(), _ptr(bias), nbias, R, H, T,
         out.data_ptr(), out.stride(0), _stream(x.device))
    return out


def _check_row_slots(row_slots, padding_start, T, device):
    if (row_slots is None) != (padding_start is None):
        raise ValueError("Reserved padding routing requires both row_slots and padding_start")
    if row_slots is None:
        return
    if (row_slots.shape != (T,) or row_slots.stride(0) != 1 or row_slots.device != device
            or row_slots.dtype not in (torch.int32, torch.int64)):
        raise ValueError("Expected one contiguous integer slot per MoE row on the same device")
    if not isinstance(padding_start, int) or padding_start <= 0:
        raise ValueError("padding_start must be a positive reserved-slot boundary")


def route_topk(logits: torch.Tensor, k: int = 8, bias: torch.Tensor | None = None,
               weights_dtype: torch.dtype | None = None, row_slots: torch.Tensor | None = None,
               padding_start: int | None = None):
    """Returns (weights [T,k], ids int64 [T,k]) like src/drama3/kernels.py:379-383.
    With row_slots/padding_start, rows whose slot is >= padding_start route with
    row 0's logits (src/drama3/moe_input.py:32-36)."""
    _require_cuda(logits, bias)
    if logits.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("router logits must be bfloat16 or float32")
    T, E = logits.shape
    _check_row_slots(row_slots, padding_start, T, logits.device)
    wdt = weights_dtype or logits.dtype
    ids = torch.empty((T, k), dtype=torch.int64, device=logits.device)
    w = torch.empty((T, k), dtype=wdt, device=logits.device)
    if bias is not None:
        bias = bias.to(torch.float32).contiguous()
    ldt = _lib.D3_DTYPE_F32 if logits.dtype == torch.float32 else _lib.D3_DTYPE_BF16
    wdt_tag = _lib.D3_DTYPE_F32 if wdt == torch.float32 else _lib.D3_DTYPE_BF16
    if row_slots is not None:
        call("d3_route_topk_rows", logits.data_ptr(), ldt, _row_stride(logits), T, E, k, _ptr(bias),
             row_slots.data_ptr(), 1 if row_slots.dtype == torch.int64 else 0, padding_start,
             ids.data_ptr(), w.data_ptr(), wdt_tag, _stream(logits.device))
    else:
        call("d3_route_topk", logits.data_ptr(), ldt, _row_stride(logits), T, E, k, _ptr(bias),
             ids.data_ptr(), w.data_ptr(), wdt_tag, _stream(logits.device))
    return w, ids


def moe_permute(topk_ids: torch.Tensor, num_experts: int, block_m: int = 16, chunked: bool = False):
    """Reference bucketing buffers (src/drama3/kernels.py:711-731):
    (counts, starts, total, sorted_ids, expert_ids, inverse_rows, active, n_active).
    chunked=True runs the multi-CTA form (used by the layer from 8192 pairs)."""
    _require_cuda(topk_ids)
    if topk_ids.dtype != torch.int64 or not topk_ids.is_contiguous():
        raise ValueError("topk_ids must be contiguous int64")
    T, k = topk_ids.shape
    P = T * k
    max_rows = -(-(P + min(P, num_experts) * (block_m - 1)) // block_m) * block_m
    max_rows = max(max_rows, block_m)
    dev = topk_ids.device
    i32 = dict(dtype=torch.int32, device=dev)
    counts = torch.empty(num_experts, **i32)
    starts = torch.empty(num_experts, **i32)
    total = torch.empty(1, **i32)
    sorted_ids = torch.empty(max_rows, **i32)
    expert_ids = torch.empty(max_rows // block_m, **i32)
    inv = torch.empty(max(P, 1), **i32)
    active = torch.empty(num_experts, **i32)
    n_active = torch.empty(1, **i32)
    if chunked:
        nbytes = ctypes.c_size_t()
        call("d3_moe_permute_scratch_size", num_experts, ctypes.byref(nbytes))
        scratch = torch.empty(nbytes.value, dtype=torch.uint8, device=dev)
        call("d3_moe_permute_chunked", topk_ids.data_ptr(), T, k, num_experts, block_m,
             counts.data_ptr(), starts.data_ptr(), total.data_ptr(), sorted_ids.data_ptr(),
             expert_ids.data_ptr(), max_rows, inv.data_ptr(), active.data_ptr(), n_active.data_ptr(),
             scratch.data_ptr(), scratch.numel(), _stream(dev))
    else:
        call("d3_moe_permute", topk_ids.data_ptr(), T, k, num_experts, block_m, counts.data_ptr(),
             starts.data_ptr(), total.data_ptr(), sorted_ids.data_ptr(), expert_ids.data_ptr(),
             max_rows, inv.data_ptr(), active.data_ptr(), n_active.data_ptr(), _stream(dev))
    return counts, starts, total, sorted_ids, expert_ids, inv[:P], active, n_active


def silu_mul(projected: torch.Tensor) -> torch.Tensor:
    _require_cuda(projected)
    rows, w2 = projected.shape
    W = w2 // 2
    out = torch.empty((rows, W), dtype=projected.dtype, device=projected.device)
    call("d3_silu_mul", projected.data_ptr(), _row_stride(projected), rows, W, out.data_ptr(),
         _stream(projected.device))
    return out


def silu_mul_quant(projected: torch.Tensor):
    _require_cuda(projected)
    rows, w2 = projected.shape
    W = w2 // 2
    q = torch.empty((rows, W), dtype=FP8, device=projected.device)
    s = torch.empty((rows, W // 128), dtype=torch.float32, device=projected.device)
    call("d3_silu_mul_quant", projected.data_ptr(), _row_stride(projected), rows, W, q.data_ptr(),
         s.data_ptr(), _stream(projected.device))
    return q, s


def combine_experts(routed: torch.Tensor, shared: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    _require_cuda(routed, shared, gate)
    T, H = routed.shape
    if not routed.is_contiguous() or not shared.is_contiguous():
        raise ValueError("routed and shared outputs must be contiguous")
    out = torch.empty_like(routed)
    call("d3_combine_experts", routed.data_ptr(), shared.data_ptr(), gate.data_ptr(), gate.stride(0),
         T, H, out.data_ptr(), _stream(routed.device))
    return out


def _norm_args(residual: torch.Tensor, weight: torch.Tensor):
    if residual.dtype != torch.bfloat16 or not residual.is_contiguous():
        raise ValueError("residual must be contiguous bf16 [T, W]")
    W = residual.shape[-1]
    if weight.numel() != W:
        raise ValueError(f"norm weight has {weight.numel()} elements, expected {W}")
    return weight.to(torch.bfloat16).contiguous()


def add_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, epsilon: float) -> torch.Tensor:
    """residual <- bf16(x + residual) in place; returns RMSNorm(residual) * (1 + weight)."""
    _require_cuda(x, residual, weight)
    w = _norm_args(residual, weight)
    if x.shape != residual.shape or x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("x must be contiguous bf16 with the residual's shape")
    out = torch.empty_like(residual)
    T, W = residual.shape
    call("d3_add_norm", x.data_ptr(), residual.data_ptr(), w.data_ptr(), float(epsilon), T, W,
         out.data_ptr(), _stream(x.device))
    return out


def combine_experts_add_norm(routed: torch.Tensor, shared: torch.Tensor, gate: torch.Tensor,
                             residual: torch.Tensor, weight: torch.Tensor, epsilon: float,
                             inverse: torch.Tensor | None = None) -> torch.Tensor:
    """residual <- bf16(fma_bf16(shared, bf16(sigmoid(gate)), routed) + residual) in
    place; returns RMSNorm(residual) * (1 + weight). With `inverse`, row t reads
    routed/shared/gate row inverse[t]."""
    _require_cuda(routed, shared, gate, residual, weight)
    w = _norm_args(residual, weight)
    if not routed.is_contiguous() or not shared.is_contiguous() or routed.shape != shared.shape:
        raise ValueError("routed and shared must be contiguous and of one shape")
    T, W = residual.shape
    if routed.shape[-1] != W:
        raise ValueError("routed/shared width differs from the residual's")
    inv = None
    if inverse is not None:
        inv = inverse.to(torch.int32).contiguous()
        if inv.numel() != T:
            raise ValueError("inverse must hold one source row per residual row")
    elif routed.shape[0] != T:
        raise ValueError("routed rows differ from residual rows (pass inverse)")
    out = torch.empty_like(residual)
    call("d3_combine_experts_add_norm", routed.data_ptr(), shared.data_ptr(), gate.data_ptr(),
         gate.stride(0), _ptr(inv), T, W, residual.data_ptr(), w.data_ptr(), float(epsilon),
         out.data_ptr(), _stream(routed.device))
    return out


def fp8_quantize_weight(weight: torch.Tensor):
    """bf16 [N,K] -> (e4m3 [Npad,K], f32 [Npad/128, K/128])."""
    _require_cuda(weight)
    if weight.dtype != torch.bfloat16 or not weight.is_contiguous():
        raise ValueError("weight must be contiguous bfloat16")
    N, K = weight.shape
    if K % 128:
        raise ValueError("Experimental dense FP8 needs a 128-aligned reduction width")
    npad = -(-N // 128) * 128
    q = torch.empty((npad, K), dtype=FP8, device=weight.device)
    s = torch.empty((npad // 128, K // 128), dtype=torch.float32, device=weight.device)
    call("d3_fp8_quantize_weight", weight.data_ptr(), N, K, q.data_ptr(), s.data_ptr(),
         _stream(weight.device))
    return q, s


def fp8_gemv(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, n: int | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """y bf16 [T,N] = x bf16 [T,K] . dequant(wq, scales)^T (weight-only FP8)."""
    _require_cuda(x, wq, scales)
    if x.dtype != torch.bfloat16:
        raise ValueError("x must be bfloat16")
    T, K = x.shape
    N = wq.shape[0] if n is None else n
    if wq.shape[1] != K or not wq.is_contiguous() or wq.dtype != FP8:
        raise ValueError("wq must be contiguous float8_e4m3fn [>=N, K]")
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=x.device)
    nbytes = ctypes.c_size_t()
    call("d3_fp8_gemv_workspace_size", T, N, K, ctypes.byref(nbytes))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=x.device)
    call("d3_fp8_gemv", x.data_ptr(), _row_stride(x), wq.data_ptr(), scales.data_ptr(), T, N, K,
         out.data_ptr(), out.stride(0), ws.data_ptr(), nbytes.value, None, _stream(x.device))
    return out


def fp8_gated_gemv(x: torch.Tensor, gate: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
                   mode: str, n: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """y bf16 [T,N] = bf16(x * bf16(act(gate))) . dequant(wq, scales)^T with
    act = silu (mode "swiglu") or sigmoid (mode "sigmoid")."""
    _require_cuda(x, gate, wq, scales)
    if x.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16:
        raise ValueError("x and gate must be bfloat16")
    if mode not in ("swiglu", "sigmoid"):
        raise ValueError("Expected swiglu or sigmoid")
    T, K = x.shape
    if tuple(gate.shape) != (T, K):
        raise ValueError("gate must have the shape of x")
    N = wq.shape[0] if n is None else n
    if wq.shape[1] != K or not wq.is_contiguous() or wq.dtype != FP8:
        raise ValueError("wq must be contiguous float8_e4m3fn [>=N, K]")
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=x.device)
    nbytes = ctypes.c_size_t()
    call("d3_fp8_gemv_workspace_size", T, N, K, ctypes.byref(nbytes))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=x.device)
    call("d3_fp8_gated_gemv", x.data_ptr(), _row_stride(x), gate.data_ptr(), _row_stride(gate),
         _lib.D3_GATE_SWIGLU if mode == "swiglu" else _lib.D3_GATE_SIGMOID, wq.data_ptr(),
         scales.data_ptr(), T, N, K, out.data_ptr(), out.stride(0), ws.data_ptr(), nbytes.value, None,
         _stream(x.device))
    return out


def set_prefill_min_tokens(t: int) -> int:
    """Token count from which the expert GEMMs run on the tcgen05 prefill
    kernel (t <= 0 restores the default); returns the previous value."""
    return int(_lib.load().d3_set_prefill_min_tokens(int(t)))


class prefill_min_tokens:
    """Context manager form of set_prefill_min_tokens."""

    def __init__(self, t: int):
        self.t = t
        self.prev = None

    def __enter__(self):
        self.prev = set_prefill_min_tokens(self.t)
        return self

    def __exit__(self, *exc):
        set_prefill_min_tokens(self.prev)
        return False


def moe_workspace(T: int, k: int, E: int, I: int, H: int, has_shared: bool, device) -> torch.Tensor:
    nbytes = ctypes.c_size_t()
    call("d3_moe_workspace_size", T, k, E, I, H, int(has_shared), ctypes.byref(nbytes))
    return torch.empty(nbytes.value, dtype=torch.uint8, device=device)


def moe_experts(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, experts,
                shared=None, workspace: torch.Tensor | None = None, status: torch.Tensor | None = None):
    """Routed (+ shared) expert outputs for given routing: (routed, shared|None)."""
    _require_cuda(x, topk_ids, topk_weights)
    if x.dtype != torch.bfloat16:
        raise ValueError("x must be bfloat16")
    ev = experts if isinstance(experts, ExpertView) else ExpertView(experts)
    sv = None if shared is None else (shared if isinstance(shared, ExpertView) else ExpertView(shared))
    T, H = x.shape
    if H != ev.H:
        raise ValueError(f"hidden size {H} != expert H {ev.H}")
    k = topk_ids.shape[1]
    if topk_ids.dtype != torch.int64 or not topk_ids.is_contiguous():
        raise ValueError("topk_ids must be contiguous int64")
    if topk_weights.dtype != torch.bfloat16:
        topk_weights = topk_weights.to(torch.bfloat16)
    topk_weights = topk_weights.contiguous()
    routed = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    shared_out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device) if sv is not None else None
    if workspace is None:
        workspace = moe_workspace(T, k, ev.E, ev.I, ev.H, sv is not None, x.device)
    call("d3_moe_experts", x.data_ptr(), _row_stride(x), topk_ids.data_ptr(), topk_weights.data_ptr(),
         T, k, ctypes.byref(ev.struct), ctypes.byref(sv.struct) if sv is not None else None,
         routed.data_ptr(), _ptr(shared_out), workspace.data_ptr(), workspace.numel(),
         _ptr(status), _stream(x.device))
    return routed, shared_out


def moe_gate_up_silu(x: torch.Tensor, topk_ids: torch.Tensor, experts, shared=None,
                     workspace: torch.Tensor | None = None,
                     status: torch.Tensor | None = None) -> torch.Tensor:
    """First stage of moe_experts: the pairs bucketed by expert, x quantised
    into expert order, gate_up + SiLU*mul + FP8 requant (the reference's
    expert_up_kernel and silu_mul_quant, src/drama3/kernels.py:290-301, 344).
    Returns the workspace that holds the activations; moe_down_combine reads
    them from it with the same routing, experts and shared expert."""
    _require_cuda(x, topk_ids)
    if x.dtype != torch.bfloat16:
        raise ValueError("x must be bfloat16")
    ev = experts if isinstance(experts, ExpertView) else ExpertView(experts)
    sv = None if shared is None else (shared if isinstance(shared, ExpertView) else ExpertView(shared))
    T, H = x.shape
    if H != ev.H:
        raise ValueError(f"hidden size {H} != expert H {ev.H}")
    if topk_ids.dtype != torch.int64 or not topk_ids.is_contiguous() or topk_ids.shape[0] != T:
        raise ValueError("topk_ids must be contiguous int64 [T, k]")
    k = topk_ids.shape[1]
    if workspace is None:
        workspace = moe_workspace(T, k, ev.E, ev.I, ev.H, sv is not None, x.device)
    call("d3_moe_gate_up_silu", x.data_ptr(), _row_stride(x), topk_ids.data_ptr(), T, k,
         ctypes.byref(ev.struct), ctypes.byref(sv.struct) if sv is not None else None,
         workspace.data_ptr(), workspace.numel(), _ptr(status), _stream(x.device))
    return workspace


def moe_down_combine(topk_weights: torch.Tensor, workspace: torch.Tensor, experts, shared=None,
                     status: torch.Tensor | None = None):
    """Second stage of moe_experts, from the workspace moe_gate_up_silu filled:
    down GEMM and the fixed-order combine (src/drama3/kernels.py:304-322).
    Returns (routed, shared|None) like moe_experts, bit for bit."""
    _require_cuda(topk_weights, workspace)
    ev = experts if isinstance(experts, ExpertView) else ExpertView(experts)
    sv = None if shared is None else (shared if isinstance(shared, ExpertView) else ExpertView(shared))
    if topk_weights.dim() != 2:
        raise ValueError("topk_weights must be [T, k]")
    T, k = topk_weights.shape
    topk_weights = topk_weights.to(torch.bfloat16).contiguous()
    routed = torch.empty((T, ev.H), dtype=torch.bfloat16, device=topk_weights.device)
    shared_out = (torch.empty((T, ev.H), dtype=torch.bfloat16, device=topk_weights.device)
                  if sv is not None else None)
    call("d3_moe_down_combine", topk_weights.data_ptr(), T, k, ctypes.byref(ev.struct),
         ctypes.byref(sv.struct) if sv is not None else None, routed.data_ptr(), _ptr(shared_out),
         workspace.data_ptr(), workspace.numel(), _ptr(status), _stream(topk_weights.device))
    return routed, shared_out


def moe_experts_fp8(q: torch.Tensor, scales: torch.Tensor, topk_ids: torch.Tensor,
                    topk_weights: torch.Tensor, experts, transposed: bool = True,
                    workspace: torch.Tensor | None = None, status: torch.Tensor | None = None):
    """Routed expert output bf16 [T,H] for already-quantised activations q e4m3
    [T,H] with group scales f32 [H/128,T] (transposed, FlashInfer's layout) or
    [T,H/128]. ids outside [0,E) contribute nothing."""
    _require_cuda(q, scales, topk_ids, topk_weights)
    if q.dtype != FP8 or q.dim() != 2 or q.stride(1) != 1:
        raise ValueError("hidden states must be float8_e4m3fn [T, H] with contiguous channels")
    if scales.dtype != torch.float32 or not scales.is_contiguous():
        raise ValueError("hidden-state scales must be contiguous float32")
    ev = experts if isinstance(experts, ExpertView) else ExpertView(experts)
    T, H = q.shape
    if H != ev.H:
        raise ValueError(f"hidden size {H} != expert H {ev.H}")
    if tuple(scales.shape) != ((H // 128, T) if transposed else (T, H // 128)):
        raise ValueError(f"hidden-state scales shape {tuple(scales.shape)} does not match T={T}, H={H}")
    if topk_ids.dtype != torch.int64 or not topk_ids.is_contiguous() or topk_ids.shape[0] != T:
        raise ValueError("topk_ids must be contiguous int64 [T, k]")
    k = topk_ids.shape[1]
    topk_weights = topk_weights.to(torch.bfloat16).contiguous()
    out = torch.empty((T, H), dtype=torch.bfloat16, device=q.device)
    if workspace is None:
        workspace = moe_workspace(T, k, ev.E, ev.I, ev.H, False, q.device)
    call("d3_moe_experts_fp8", q.data_ptr(), q.stride(0), scales.data_ptr(), int(transposed),
         topk_ids.data_ptr(), topk_weights.data_ptr(), T, k, ctypes.byref(ev.struct), out.data_ptr(),
         workspace.data_ptr(), workspace.numel(), _ptr(status), _stream(q.device))
    return out


def _row_map(t, name, device):
    if t is None:
        return None
    if t.dtype != torch.int64 or t.dim() != 1 or t.stride(0) != 1 or t.device != device:
        raise ValueError(f"{name} must be a contiguous int64 vector on the layer's device")
    return t


def moe_layer(x: torch.Tensor, router_weight: torch.Tensor, experts, shared, k: int = 8,
              router_bias: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
              out: torch.Tensor | None = None, return_routing: bool = False,
              status: torch.Tensor | None = None, residual: torch.Tensor | None = None,
              norm_weight: torch.Tensor | None = None, norm_eps: float = 1e-6,
              keep: torch.Tensor | None = None, inverse: torch.Tensor | None = None,
              row_slots: torch.Tensor | None = None, padding_start: int | None = None):
    """Whole MoE layer: out = routed + bf16(shared * bf16(sigmoid(gate))).
    With `residual` and `norm_weight` the layer exit is fused in: residual is
    updated in place with the bf16-fma combine (combine_experts_add_norm) and
    out = RMSNorm(residual) * (1 + norm_weight).

    Row maps of the mixed decode + packed-prefill call
    (src/drama3/mixed_model.py:193-246): `keep` (int64 [T]) runs the MoE over
    x[keep] without materialising it (T = len(keep)); `inverse` (int64
    [T_out], fused exit only) makes residual row t take MoE row inverse[t];
    `row_slots` (int32/int64 [T]) with `padding_start` routes rows whose slot
    is >= padding_start with row 0's logits (src/drama3/moe_input.py:32-36)."""
    _require_cuda(x, router_weight, router_bias)
    ev = experts if isinstance(experts, ExpertView) else ExpertView(experts)
    sv = shared if isinstance(shared, ExpertView) else ExpertView(shared)
    H = x.shape[1]
    keep = _row_map(keep, "keep", x.device)
    inverse = _row_map(inverse, "inverse", x.device)
    T = len(keep) if keep is not None else x.shape[0]
    _check_row_slots(row_slots, padding_start, T, x.device)
    if inverse is not None and residual is None:
        raise ValueError("an inverse row map needs the fused exit (residual and norm_weight)")
    T_out = len(inverse) if inverse is not None else T
    if router_weight.shape != (ev.E + 1, H) or router_weight.dtype != torch.bfloat16:
        raise ValueError("router_weight must be bf16 [E+1, H] (router rows + shared-gate row)")
    if out is None:
        out = torch.empty((T_out, H), dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = moe_workspace(T, k, ev.E, ev.I, ev.H, True, x.device)
    ids = torch.empty((T, k), dtype=torch.int64, device=x.device) if return_routing else None
    wts = torch.empty((T, k), dtype=torch.bfloat16, device=x.device) if return_routing else None
    if router_bias is not None:
        router_bias = router_bias.to(torch.float32).contiguous()
    nw = None
    if residual is not None:
        if norm_weight is None:
            raise ValueError("the fused layer exit needs norm_weight with residual")
        _require_cuda(residual, norm_weight)
        nw = _norm_args(residual, norm_weight)
        if residual.shape != (T_out, H):
            raise ValueError(f"residual must be [{T_out}, H]")
    if keep is not None or inverse is not None or row_slots is not None:
        rows = D3Rows(_ptr(keep), x.shape[0], _ptr(inverse), T_out, _ptr(row_slots),
                      1 if row_slots is not None and row_slots.dtype == torch.int64 else 0,
                      padding_start or 0)
        call("d3_moe_layer_rows", x.data_ptr(), _row_stride(x), router_weight.data_ptr(),
             _ptr(router_bias), T, k, ctypes.byref(ev.struct), ctypes.byref(sv.struct),
             ctypes.byref(rows), _ptr(residual), _ptr(nw), float(norm_eps), out.data_ptr(), _ptr(ids),
             _ptr(wts), workspace.data_ptr(), workspace.numel(), _ptr(status), _stream(x.device))
    elif residual is not None:
        call("d3_moe_layer_add_norm", x.data_ptr(), _row_stride(x), router_weight.data_ptr(),
             _ptr(router_bias), T, k, ctypes.byref(ev.struct), ctypes.byref(sv.struct),
             residual.data_ptr(), nw.data_ptr(), float(norm_eps), out.data_ptr(), _ptr(ids), _ptr(wts),
             workspace.data_ptr(), workspace.numel(), _ptr(status), _stream(x.device))
    else:
        call("d3_moe_layer", x.data_ptr(), _row_stride(x), router_weight.data_ptr(), _ptr(router_bias),
             T, k, ctypes.byref(ev.struct), ctypes.byref(sv.struct), out.data_ptr(), _ptr(ids), _ptr(wts),
             workspace.data_ptr(), workspace.numel(), _ptr(status), _stream(x.device))
    if return_routing:
        return out, ids, wts
    return out
