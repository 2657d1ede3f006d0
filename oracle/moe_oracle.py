"""CPU oracle of the Drama 3 FP8 MoE hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of the reference operators in
src/drama3/ (cited per function). It is the checker for the CUDA kernels and
the timed CPU baseline; it is never imported by the product package
(d3moe), whose operators fail loudly when libd3moe.so is missing.

Pinning: every function below is checked against golden vectors produced by
running the reference's own Triton kernels (Triton interpreter, CPU) —
tests/golden/make_golden.py and tests/test_oracle_golden.py.

Number formats: bf16 tensors are float32 arrays holding bf16-representable
values; e4m3 tensors are uint8 arrays of OCP FP8 E4M3 ("fn") bytes.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32

# ------------------------------------------------------------------ formats --


def _e4m3_table() -> np.ndarray:
    """Value of each E4M3 byte (OCP FP8 E4M3: bias 7, no infinities,
    S.1111.111 = NaN, max finite 448)."""
    vals = np.zeros(256, dtype=np.float64)
    for b in range(256):
        s, e, m = b >> 7, (b >> 3) & 15, b & 7
        if e == 15 and m == 7:
            v = np.nan
        elif e == 0:
            v = (m / 8.0) * 2.0 ** -6
        else:
            v = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        vals[b] = -v if s else v
    return vals


E4M3_VALUES = _e4m3_table()
E4M3_F32 = E4M3_VALUES.astype(np.float32)
_POS = E4M3_VALUES[:127]  # codes 0..126, ascending, finite


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    return E4M3_F32[np.asarray(b, dtype=np.uint8)]


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """float32 -> E4M3 byte, round-to-nearest-even, saturating at +-448
    (the semantics of cvt.rn.satfinite.e4m3x2.f32 used when Triton stores
    fp32 into an fp8e4nv tensor)."""
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v).astype(np.float64)
    hi = np.searchsorted(_POS, a, side="left")
    hi = np.minimum(hi, 126)
    lo = np.maximum(hi - 1, 0)
    d_lo = a - _POS[lo]
    d_hi = _POS[hi] - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((hi & 1) == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(a >= _POS[126], 126, code)  # satfinite
    code = np.where(a <= 0, 0, code)
    code = code.astype(np.uint8) | np.where(np.signbit(v), 0x80, 0).astype(np.uint8)
    code = np.where(np.isnan(v), 0x7F, code).astype(np.uint8)
    return code


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bfloat16, returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), out).astype(np.float32)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_to_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


# ------------------------------------------------------ activation quantiser --


def quant_act_values(x: np.ndarray, group: int = 128):
    """The fp32 values the activation quantiser stores, before the e4m3 store
    conversion: src/drama3/moe_input.py:24-27, scale = max(amax, 1e-10)/448,
    q = clamp(x / scale, -448, 448) (IEEE fp32 division).
    Returns (q f32 [T,H], scales f32 [T, H/group])."""
    x = np.asarray(x, dtype=np.float32)
    T, H = x.shape
    g = x.reshape(T, H // group, group)
    amax = np.abs(g).max(axis=2)
    scale = (np.maximum(amax, F32(1e-10)) / F32(448.0)).astype(np.float32)
    q = np.clip(g / scale[:, :, None], F32(-448.0), F32(448.0)).astype(np.float32)
    return q.reshape(T, H), scale


def quant_act_fp8(x: np.ndarray, group: int = 128):
    """Per-row, per-128-column FP8 quantisation (moe_input.py:24-27): the
    values of quant_act_values stored as e4m3 (round-to-nearest-even).
    Returns (q bytes [T,H], scales f32 [T, H/group])."""
    q, scale = quant_act_values(x, group)
    return e4m3_encode(q), scale


def prepare_moe_input(x, router, row_slots=None, padding_start=None, values=False):
    """src/drama3/moe_input.py:8-79: (q [T,H], scales [H/128, T], logits f32
    [T,E]); rows with slot >= padding_start take row 0's router logits.
    values=True returns q as the fp32 pre-store values."""
    q, s = quant_act_values(x) if values else quant_act_fp8(x)
    logits = np.asarray(router, dtype=np.float32).copy()
    if row_slots is not None and padding_start:
        pad = np.asarray(row_slots) >= padding_start
        logits[pad] = logits[0]
    return q, np.ascontiguousarray(s.T), logits


# --------------------------------------------------------- router projection --


def router_logits(x, w, bias=None, nbias=None):
    """bf16 logits = x . w^T in the fixed fp32 order of the CUDA-core router
    kernels (used below 256 tokens): lane l (of 32) accumulates
    k = 256*i + 8*l + j sequentially (i, then j = 0..7), then lanes combine by
    xor-butterfly 16, 8, 4, 2, 1; + bias; rounded to bf16. Replaces
    linear(x, layer.gate.weight) (src/drama3/model.py:496-504) with a
    reproducible order. The tensor-core router used from 256 tokens sums in
    the hardware's order and is held to one bf16 ulp of this value (or the
    fp32 noise floor where the sum cancels to near zero)."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    T, H = x.shape
    R = w.shape[0]
    acc = np.zeros((T, R, 32), dtype=np.float32)
    lanes = np.arange(32)
    for i in range((H + 255) // 256):
        for j in range(8):
            k = 256 * i + 8 * lanes + j
            valid = k < H
            kk = np.where(valid, k, 0)
            prod = (x[:, None, kk] * w[None, :, kk]).astype(np.float32)
            prod = np.where(valid[None, None, :], prod, F32(0.0))
            acc = (acc + prod).astype(np.float32)
    for o in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, :, lanes ^ o]).astype(np.float32)
    out = acc[:, :, 0]
    if bias is not None:
        b = np.zeros(R, dtype=np.float32)
        nb = len(bias) if nbias is None else nbias
        b[:nb] = np.asarray(bias, dtype=np.float32)[:nb]
        out = (out + b[None, :]).astype(np.float32)
    return bf16_round(out)


# -------------------------------------------------------------------- route --


def route_keys(v: np.ndarray) -> np.ndarray:
    """Order keys: sign-flipped fp32 bits (high word), inverted column (low
    word). For bf16 logits this orders exactly like the reference's
    (ordered & 0xFFFF0000) | (65535 - col) (src/drama3/kernels.py:365-369)."""
    bits = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32)
    ordered = bits ^ np.where(bits & 0x80000000, np.uint32(0xFFFFFFFF), np.uint32(0x80000000))
    cols = np.arange(v.shape[-1], dtype=np.uint64)
    return (ordered.astype(np.uint64) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - cols)


def route(logits, k: int = 8, bias=None, row_slots=None, padding_start=None):
    """src/drama3/kernels.py:360-383: fp32 softmax over all experts, top-k by
    logit (ties to the lower expert id), weights renormalised over the picks.
    With row_slots/padding_start, rows whose slot is >= padding_start take
    row 0's logits (src/drama3/moe_input.py:32-36).
    Returns (weights f32 [T,k], ids int64 [T,k]); callers round weights to the
    logits dtype (bf16 in the reference)."""
    v = np.asarray(logits, dtype=np.float32)
    if row_slots is not None and padding_start:
        v = np.where((np.asarray(row_slots) >= padding_start)[:, None], v[0:1], v)
    if bias is not None:
        v = (v + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    keys = route_keys(v)  # unique per row (the column is part of the key)
    ids = np.argsort(keys, axis=1)[:, ::-1][:, :k].astype(np.int64)
    mx = v.max(axis=1, keepdims=True)
    denom = np.exp(v - mx).astype(np.float32).sum(axis=1, keepdims=True, dtype=np.float32)
    p = (np.exp(np.take_along_axis(v, ids, axis=1) - mx).astype(np.float32) / denom).astype(np.float32)
    wts = (p / p.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return wts, ids


# ------------------------------------------------------------------ permute --


def moe_permute(ids, num_experts: int, block_m: int):
    """src/drama3/kernels.py:658-699 with the buffers of kernels.py:711-731.

    Pairs p = t*k + r. counts[e]; starts = exclusive cumsum of counts padded to
    block_m; total = their sum; sorted_ids[starts[e] + i] = i-th pair (ascending)
    routed to e, padding slots = P (sentinel); expert_ids[starts[e]/block_m + b]
    = e. Slots past `total` are left unspecified by the reference; this oracle
    returns only [0, total) and [0, total/block_m)."""
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    P = ids.size
    counts = np.bincount(ids[(ids >= 0) & (ids < num_experts)], minlength=num_experts).astype(np.int32)
    padded = (counts + block_m - 1) // block_m * block_m
    starts = (np.cumsum(padded) - padded).astype(np.int32)
    total = int(padded.sum())
    sorted_ids = np.full(total, P, dtype=np.int32)
    expert_ids = np.zeros(total // block_m, dtype=np.int32)
    for e in range(num_experts):
        pairs = np.nonzero(ids == e)[0]
        sorted_ids[starts[e]: starts[e] + len(pairs)] = pairs
        expert_ids[starts[e] // block_m: (starts[e] + padded[e]) // block_m] = e
    return counts, starts, total, sorted_ids, expert_ids


# ---------------------------------------------------------- expert weights --


def dequant_blocks(wq: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """e4m3 [R, C] with f32 scales [R/128, C/128] -> f32 [R, C]
    (the block dequantisation of scripts/diagnostic_mxfp8_moe.py:36-43)."""
    R, C = wq.shape
    w = e4m3_decode(wq).reshape(R // 128, 128, C // 128, 128)
    return (w * scales[:, None, :, None]).astype(np.float32).reshape(R, C)


def dequant_rows(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """e4m3 [T, C] with per-row 1x128 scales [T, C/128] -> f32."""
    T, C = q.shape
    return (e4m3_decode(q).reshape(T, C // 128, 128) * scales[:, :, None]).astype(np.float32).reshape(T, C)


def quantize_weight_blocks(w, min_scale: float = 1e-8, values: bool = False):
    """src/drama3/experimental_fp8.py:10-18 (and register, :45-53): rows padded
    to a multiple of 128 with zeros; scale = max(amax, 1e-8)/448 per 128x128
    block; q = e4m3(w / scale). Returns (q [Npad,K], scales [Npad/128, K/128]);
    values=True returns q as the fp32 pre-store values."""
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    npad = -(-N // 128) * 128
    wp = np.zeros((npad, K), dtype=np.float32)
    wp[:N] = w
    b = wp.reshape(npad // 128, 128, K // 128, 128)
    amax = np.abs(b).max(axis=(1, 3))
    scale = (np.maximum(amax, F32(min_scale)) / F32(448.0)).astype(np.float32)
    qv = (b / scale[:, None, :, None]).astype(np.float32).reshape(npad, K)
    return (qv if values else e4m3_encode(qv)), scale


# ------------------------------------------------------------ expert math --


def silu_bf16(g: np.ndarray) -> np.ndarray:
    g = np.asarray(g, dtype=np.float32)
    return bf16_round((g * (F32(1.0) / (F32(1.0) + np.exp(-g)))).astype(np.float32))


def silu_mul(projected):
    """src/drama3/kernels.py:386-402: bf16(bf16(silu(gate)) * up)."""
    p = np.asarray(projected, dtype=np.float32)
    W = p.shape[1] // 2
    return bf16_round((silu_bf16(p[:, :W]) * p[:, W:]).astype(np.float32))


def silu_mul_quant(projected):
    """Fish silu_mul_quant_kernel via quantize_groups(·, gate_up, I)
    (called at src/drama3/kernels.py:344, :748): a = bf16(silu(gate)) * up in
    fp32, then the 1x128 activation quantiser of moe_input.py:24-27."""
    p = np.asarray(projected, dtype=np.float32)
    W = p.shape[1] // 2
    a = (silu_bf16(p[:, :W]) * p[:, W:]).astype(np.float32)
    return quant_act_fp8(a)


def expert_gate_up(q, sx, w13, s13, ids):
    """src/drama3/kernels.py:290-301: for pair (t, r) with expert e = ids[t,r],
    gu[t*k+r, n] = sum_k W13[e,n,k]*S13[e,n/128,k/128]*q[t,k]*sx[t,k/128] in
    fp32, stored bf16. w13/s13 may be dicts {expert: array}."""
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    act = dequant_rows(q, sx)
    n2 = w13[int(ids.flat[0])].shape[0]
    out = np.zeros((T * k, n2), dtype=np.float32)
    for e in np.unique(ids):
        wd = dequant_blocks(w13[int(e)], s13[int(e)])
        pairs = np.nonzero(ids.reshape(-1) == e)[0]
        out[pairs] = act[pairs // k] @ wd.T
    return bf16_round(out)


def expert_down_rows(a, sa, w2, s2, ids):
    """Per-pair fp32 down projection d[p, n] = sum_k W2[e,n,k]*S2[..]*a[p,k]*sa[p,k/128]."""
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    act = dequant_rows(a, sa)
    H = w2[int(ids[0])].shape[0]
    out = np.zeros((ids.size, H), dtype=np.float32)
    for e in np.unique(ids):
        wd = dequant_blocks(w2[int(e)], s2[int(e)])
        pairs = np.nonzero(ids == e)[0]
        out[pairs] = act[pairs] @ wd.T
    return out


def expert_down_combine(a, sa, w2, s2, ids, weights, skip=None, rows_bf16=False):
    """src/drama3/kernels.py:304-322: y[t] = bf16(sum_r w[t,r] * down_r) with
    fp32 accumulation (rank order r = 0..k-1); pairs marked in `skip` [T,k]
    are left out of the sum. rows_bf16: each down row is rounded to bf16
    before the sum (the tcgen05 prefill path's intermediate rows)."""
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    d = expert_down_rows(a, sa, w2, s2, ids).reshape(T, k, -1)
    if rows_bf16:
        d = bf16_round(d)
    w = np.asarray(weights, dtype=np.float32)
    acc = np.zeros((T, d.shape[2]), dtype=np.float32)
    for r in range(k):
        term = (acc + d[:, r] * w[:, r: r + 1]).astype(np.float32)
        acc = term if skip is None else np.where(skip[:, r: r + 1], acc, term)
    return bf16_round(acc)


def combine_experts(routed, shared, gate):
    """src/drama3/kernels.py:427-445: routed + bf16(shared * bf16(sigmoid(gate)))."""
    g = np.asarray(gate, dtype=np.float32).reshape(-1, 1)
    sg = bf16_round((F32(1.0) / (F32(1.0) + np.exp(-g))).astype(np.float32))
    weighted = bf16_round((np.asarray(shared, dtype=np.float32) * sg).astype(np.float32))
    return bf16_round((np.asarray(routed, dtype=np.float32) + weighted).astype(np.float32))


def bf16_fma(a, b, c):
    """PTX fma.rn.bf16: a*b + c computed exactly, rounded once to bf16. For
    bf16 operands the exact value fits a float64 (a*b has at most 16
    significant bits)."""
    exact = (np.asarray(a, np.float64) * np.asarray(b, np.float64)) + np.asarray(c, np.float64)
    return bf16_round(exact)


def _rms_scale(value, weight, eps):
    """value * rsqrt(mean(value^2) + eps) * (1 + weight), fp32 (the norm half of
    src/drama3/kernels.py:413-415 and :478-480)."""
    v = np.asarray(value, dtype=np.float32)
    ms = (np.sum(v * v, axis=-1, dtype=np.float32) / F32(v.shape[-1])).astype(np.float32)
    r = (F32(1.0) / np.sqrt((ms + F32(eps)).astype(np.float32))).astype(np.float32)
    out = (v * r[:, None]).astype(np.float32)
    out = (out * (F32(1.0) + np.asarray(weight, dtype=np.float32))[None, :]).astype(np.float32)
    return bf16_round(out)


def add_norm(x, residual, weight, eps):
    """src/drama3/kernels.py:405-423 (add_norm_kernel): residual <- bf16(x +
    residual) (fp32 add), out = bf16(rmsnorm(residual) * (1 + weight)).
    Returns (out, new_residual)."""
    value = bf16_round((np.asarray(x, np.float32) + np.asarray(residual, np.float32)).astype(np.float32))
    return _rms_scale(value, weight, eps), value


def combine_experts_add_norm(routed, shared, gate, residual, weight, eps, inverse=None):
    """src/drama3/kernels.py:448-499 (and the _inverse form :502-556): combined =
    fma.rn.bf16(shared, bf16(sigmoid(gate)), routed) on the (optionally
    inverse-gathered) rows, residual <- bf16(combined + residual) (fp32 add),
    out = bf16(rmsnorm(residual) * (1 + weight)). Returns (out, new_residual)."""
    routed = np.asarray(routed, np.float32)
    shared = np.asarray(shared, np.float32)
    g = np.asarray(gate, dtype=np.float32).reshape(-1)
    if inverse is not None:
        inv = np.asarray(inverse).reshape(-1)
        routed, shared, g = routed[inv], shared[inv], g[inv]
    sg = bf16_round((F32(1.0) / (F32(1.0) + np.exp(-g))).astype(np.float32))
    combined = bf16_fma(shared, sg[:, None], routed)
    value = bf16_round((combined + np.asarray(residual, np.float32)).astype(np.float32))
    return _rms_scale(value, weight, eps), value


def gated_input(x, gate, mode):
    """src/drama3/fused_projection.py:22-29: a = bf16(silu(g)) ("swiglu") or
    bf16(sigmoid(g)) ("sigmoid"), sigmoid(g) = 1 / (1 + exp(-g)) in fp32;
    returns bf16(x * a), the input the projection multiplies."""
    g = np.asarray(gate, dtype=np.float32)
    sg = (F32(1.0) / (F32(1.0) + np.exp(-g))).astype(np.float32)
    a = bf16_round((g * sg).astype(np.float32) if mode == "swiglu" else sg)
    return bf16_round((np.asarray(x, np.float32) * a).astype(np.float32))


def fp8_gemv(x, wq, scales, n=None):
    """src/drama3/experimental_fp8.py:21-29 (_gemv): y = sum_k w*scale*x with
    bf16 activations (no activation quantisation), stored bf16. The sum is
    taken in float64 so the oracle returns the correctly rounded value that
    any fp32 summation order approximates."""
    wd = dequant_blocks(np.asarray(wq), np.asarray(scales))
    if n is not None:
        wd = wd[:n]
    y = np.asarray(x, dtype=np.float64) @ wd.T.astype(np.float64)
    return bf16_round(y.astype(np.float32))


# ------------------------------------------------------------ whole layer --


class Experts:
    """Expert container with the reference's layout (kernels.py:336-350):
    w13 [E,2I,H] e4m3 bytes (rows [gate|up]), s13 [E,2I/128,H/128] f32,
    w2 [E,H,I] e4m3 bytes, s2 [E,H/128,I/128] f32."""

    def __init__(self, w13, s13, w2, s2):
        self.w13, self.s13, self.w2, self.s2 = w13, s13, w2, s2


def moe_experts(x, ids, weights, ex: Experts, shared: Experts | None = None, rows_bf16=False):
    """Routed (+ shared) experts for given routing, the arithmetic of
    small_batch_moe / native_moe (src/drama3/kernels.py:325-357, 702-779) with
    the shared expert as an always-selected expert of weight 1. rows_bf16
    restates the tcgen05 prefill path, whose per-expert down rows are bf16.
    Returns (routed bf16 [T,H], shared bf16 [T,H] or None)."""
    x = np.asarray(x, dtype=np.float32)
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    q, sx = quant_act_fp8(x)
    gu = expert_gate_up(q, sx, ex.w13, ex.s13, ids)
    a, sa = silu_mul_quant(gu)
    routed = expert_down_combine(a, sa, ex.w2, ex.s2, ids, weights, rows_bf16=rows_bf16)
    sh = None
    if shared is not None:
        sid = np.zeros((T, 1), dtype=np.int64)
        gus = expert_gate_up(q, sx, shared.w13, shared.s13, sid)
        a2, sa2 = silu_mul_quant(gus)
        sh = bf16_round(expert_down_rows(a2, sa2, shared.w2, shared.s2, sid))
    return routed, sh


def moe_experts_q(q, sx, ids, weights, ex: Experts, rows_bf16=False):
    """Routed experts over already-quantised activations (q e4m3 bytes [T,H],
    sx f32 [T,H/128]): the expert arithmetic of moe_experts after its input
    quantisation, the operands FlashInfer's trtllm_fp8_block_scale_moe gets
    (src/drama3/model.py:544-580). Pairs whose id is outside [0, E) contribute
    nothing. Returns routed bf16 [T,H]."""
    ids = np.asarray(ids, dtype=np.int64)
    E = len(ex.w13)
    valid = (ids >= 0) & (ids < E)
    w = np.where(valid, np.asarray(weights, np.float32), F32(0.0)).astype(np.float32)
    safe = np.where(valid, ids, 0)
    gu = expert_gate_up(np.asarray(q), np.asarray(sx, np.float32), ex.w13, ex.s13, safe)
    a, sa = silu_mul_quant(gu)
    return expert_down_combine(a, sa, ex.w2, ex.s2, safe, w, skip=~valid, rows_bf16=rows_bf16)


def moe_layer(x, router_w, ex: Experts, shared: Experts, k: int = 8, bias=None, rows_bf16=False):
    """DramaModel.moe (src/drama3/model.py:485-541) for one FP8 layer: router
    projection over [E+1, H] (rows 0..E-1 router, row E shared-expert gate,
    model.py:236-245), top-k routing, routed + shared experts, combine.
    Returns (out bf16 [T,H], ids, weights bf16)."""
    E = router_w.shape[0] - 1
    logits = router_logits(x, router_w, bias, nbias=E)
    w, ids = route(logits[:, :E], k)
    w = bf16_round(w)
    routed, sh = moe_experts(x, ids, w, ex, shared, rows_bf16=rows_bf16)
    out = combine_experts(routed, sh, logits[:, E])
    return out, ids, w


def moe_layer_rows(x, router_w, ex: Experts, shared: Experts, residual, norm_weight, eps=1e-6,
                   k: int = 8, keep=None, inverse=None, row_slots=None, padding_start=None,
                   rows_bf16=False):
    """The mixed decode + packed-prefill layer step (src/drama3/mixed_model.py:
    193-246): moe_parts over x[keep] (model.py:490-518) with the padding-router
    rule on row_slots (moe_input.py:32-36), then combine_experts_add_norm or its
    _inverse form (kernels.py:448-556). Returns (out, residual_out, ids,
    weights) in float32 holding bf16 values."""
    x = np.asarray(x, dtype=np.float32)
    xk = x if keep is None else x[np.asarray(keep)]
    E = router_w.shape[0] - 1
    logits = router_logits(xk, router_w)
    w, ids = route(logits[:, :E], k, row_slots=row_slots, padding_start=padding_start)
    w = bf16_round(w)
    routed, sh = moe_experts(xk, ids, w, ex, shared, rows_bf16=rows_bf16)
    out, res = combine_experts_add_norm(routed, sh, logits[:, E:E + 1], residual, norm_weight, eps,
                                        inverse=inverse)
    return out, res, ids, w


# --------------------------------------------------------- synthetic data --


def hash_uniform(seed: int, shape, offset: int = 0) -> np.ndarray:
    """Deterministic uniform [-1, 1) floats from a splitmix64 hash of the flat
    index — identical on every machine and numpy version."""
    n = int(np.prod(shape))
    idx = np.arange(n, dtype=np.uint64) + np.uint64(offset)
    z = idx + np.uint64((seed * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    z = z ^ (z >> np.uint64(31))
    u = (z >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    return (2.0 * u - 1.0).astype(np.float32).reshape(shape)


def synth_expert(seed: int, expert: int, rows: int, cols: int, amp: float = 0.04):
    """One expert matrix: hashed uniform values in [-amp, amp) quantised with
    the 128x128 block quantiser (scale = amax/448). Returns (bytes, scales)."""
    w = hash_uniform(seed, (rows, cols), offset=expert * rows * cols) * F32(amp)
    return quantize_weight_blocks(w)
