"""Generate golden vectors by running the REFERENCE's own Triton kernels.

The reference (src/drama3/*.py of david6666666/drama-3-single-b300-inference)
is pure Python/Triton. Its kernels execute on the CPU under the Triton
interpreter (TRITON_INTERPRET=1), so this script imports them from a local
checkout and records their exact outputs. The kernels hard-code the Drama 3
geometry (H=2048, E=256, I=512, top-8), so every fixture here uses it.

Inputs are small and stored in the fixtures; large expert weights are
regenerated deterministically from oracle.moe_oracle.synth_expert (a hash of
the element index), and only the experts the fixture routes to are filled in
(the reference kernels read only those).

Down-conversions: the Triton 3.6 interpreter converts fp32 -> bf16 by
truncation and fp32 -> float8e4nv without the mantissa carry into the
exponent (-1.94 becomes -1.0), while compiled Triton on the GPU rounds to
nearest-even (cvt.rn.bf16.f32, cvt.rn.satfinite.e4m3x2.f32). Up-conversions
(loads of bf16/fp8) are exact. This script therefore replaces the
interpreter's float down-conversion routine (a tool, not reference code) with
torch's nearest-even casts, so interpreted kernels round like compiled ones.
Where a reference kernel stores fp8 (prepare_kernel's Q, _quantize's Q) the
same kernel is also launched with an fp32 destination and the exact
pre-conversion values are recorded ("*_qf32").

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_golden.py --reference <path-to-reference-checkout>
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import moe_oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent
H, E, I, K = 2048, 256, 512, 8
WSEED_UP, WSEED_DOWN = 11, 12


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def fill_experts(experts, rows, cols, seed):
    """Zero weight tensor [E, rows, cols] with the selected experts filled."""
    w = torch.zeros((E, rows, cols), dtype=torch.uint8)
    s = torch.ones((E, rows // 128, cols // 128), dtype=torch.float32)
    for e in experts:
        q, sc = O.synth_expert(seed, int(e), rows, cols)
        w[int(e)] = torch.from_numpy(q)
        s[int(e)] = torch.from_numpy(sc)
    return w.view(torch.float8_e4m3fn), s


def patch_interpreter_rounding() -> None:
    """Make the interpreter's fp32 down-conversions round to nearest-even."""
    import triton.language as tl
    from triton.runtime import interpreter

    original = interpreter._convert_float
    targets = {
        tl.bfloat16: (torch.bfloat16, np.uint16),
        tl.float16: (torch.float16, np.uint16),
        tl.float8e4nv: (torch.float8_e4m3fn, np.uint8),
    }

    def convert(input, input_dtype, output_dtype, rounding_mode):
        if input_dtype == tl.float32 and output_dtype in targets:
            tdt, udt = targets[output_dtype]
            src = torch.from_numpy(np.frombuffer(input.tobytes(), dtype=np.float32).copy())
            if tdt == torch.float8_e4m3fn:  # satfinite, NaN kept
                src = torch.where(torch.isnan(src), src, src.clamp(-448.0, 448.0))
            out = src.to(tdt).view(torch.uint8 if udt == np.uint8 else torch.int16).numpy().view(udt)
            return out.reshape(np.shape(input))
        return original(input, input_dtype, output_dtype, rounding_mode)

    interpreter._convert_float = convert


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    patch_interpreter_rounding()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    from drama3 import experimental_fp8, kernels, moe_atomic, moe_input  # noqa: E402

    rng = np.random.default_rng(20261201)

    def prepare(x, router, row_slots=None, padding_start=None):
        """prepare_moe_input (moe_input.py:40-79) with an fp32 Q destination."""
        T = len(x)
        q = torch.empty(x.shape, dtype=torch.float32)
        scales = torch.empty((16, T), dtype=torch.float32)
        logits = torch.empty(router.shape, dtype=torch.float32)
        moe_input.prepare_kernel[(T,)](x, router, q, scales, logits, row_slots, T, x.stride(0),
                                       router.stride(0), padding_start or 0, num_warps=4)
        return q, scales, logits

    def e4m3(q_f32: torch.Tensor) -> np.ndarray:
        return bits(q_f32.to(torch.float8_e4m3fn))

    # ---- prepare_moe_input: magnitudes and strides (scripts/validate_moe_input.py:27-36)
    prep = {}
    for strided in (False, True):
        for mi, mag in enumerate((0.0, 1e-12, 1.0, 1000.0)):
            T = 12
            store = bf16(rng.standard_normal((T, 4096 if strided else 2048)) * mag)
            x = store[:, :2048]
            rstore = bf16(rng.standard_normal((T, 1408 if strided else 256)))
            router = rstore[:, :256]
            q, s, lg = prepare(x, router)
            key = f"s{int(strided)}_m{mi}"
            prep[key + "_x"] = bits(x.contiguous())
            prep[key + "_router"] = bits(router.contiguous())
            prep[key + "_qf32"] = bits(q)
            prep[key + "_q"] = e4m3(q)
            prep[key + "_scales"] = bits(s)
            prep[key + "_logits"] = bits(lg)
    T = 6
    x = bf16(rng.standard_normal((T, 2048)))
    router = bf16(rng.standard_normal((T, 256)))
    slots = torch.tensor([0, 5, 40, 2, 33, 63], dtype=torch.int64)
    q, s, lg = prepare(x, router, row_slots=slots, padding_start=32)
    prep.update(pad_x=bits(x), pad_router=bits(router), pad_slots=slots.numpy(), pad_start=np.int64(32),
                pad_qf32=bits(q), pad_q=e4m3(q), pad_scales=bits(s), pad_logits=bits(lg))
    np.savez_compressed(OUT / "prepare_moe_input.npz", **prep)

    # ---- route: random rows plus ties, zeros, equal rows (kernels.py:360-383)
    lg = rng.standard_normal((16, 256)).astype(np.float32)
    lg[1, [5, 7, 100]] = 4.0                      # three-way tie at the top
    lg[2, :] = 0.5                                # all equal
    lg[3, :] = 0.0
    lg[3, 10] = -0.0
    lg[3, 200] = 1e-3
    lg[4, :] = -30.0
    lg[4, [250, 3, 77, 128, 9, 64, 31, 200, 1]] = -1.0  # tie across the top-8 boundary
    lg[5] *= 40.0                                 # peaked softmax
    logits = bf16(lg)
    w, ids = kernels.route(logits)
    np.savez_compressed(OUT / "route.npz", logits=bits(logits), ids=ids.numpy(), weights=bits(w))

    # ---- bucketing (kernels.py:658-699, buffers :711-731)
    perm = {}
    for T in (1, 5, 37):
        for bm in (16, 64):
            lgt = bf16(rng.standard_normal((T, 256)))
            _, ids = kernels.route(lgt)
            pairs = T * 8
            max_rows = -(-(pairs + min(pairs, 256) * (bm - 1)) // bm) * bm
            counts = torch.empty(256, dtype=torch.int32)
            starts = torch.empty_like(counts)
            total = torch.empty(1, dtype=torch.int32)
            sorted_ids = torch.full((max_rows,), -7, dtype=torch.int32)
            expert_ids = torch.full((max_rows // bm,), -7, dtype=torch.int32)
            import triton

            kernels.expert_counts_kernel[(256,)](ids, counts, pairs, triton.next_power_of_2(pairs))
            kernels.expert_offsets_kernel[(1,)](counts, starts, total, bm)
            kernels.expert_scatter_kernel[(256,)](
                ids, counts, starts, sorted_ids, expert_ids, pairs,
                triton.next_power_of_2(pairs), triton.next_power_of_2(triton.cdiv(T, bm)), bm)
            tot = int(total.item())
            key = f"t{T}_bm{bm}"
            perm[key + "_ids"] = ids.numpy()
            perm[key + "_counts"] = counts.numpy()
            perm[key + "_starts"] = starts.numpy()
            perm[key + "_total"] = np.int64(tot)
            perm[key + "_sorted"] = sorted_ids.numpy()[:tot]
            perm[key + "_experts"] = expert_ids.numpy()[: tot // bm]
    np.savez_compressed(OUT / "permute.npz", **perm)

    # ---- small-batch expert path: up GEMV, silu_mul, down GEMV + combine
    T = 3
    x = bf16(rng.standard_normal((T, 2048)))
    lgt = bf16(rng.standard_normal((T, 256)))
    w, ids = kernels.route(lgt)
    sel = np.unique(ids.numpy())
    w13, s13 = fill_experts(sel, 2 * I, H, WSEED_UP)
    w2, s2 = fill_experts(sel, H, I, WSEED_DOWN)
    xq, xs = O.quant_act_fp8(x.float().numpy())  # == Fish quantize_groups (validate_moe_input.py)
    xq_t = torch.from_numpy(xq).view(torch.float8_e4m3fn)
    xs_t = torch.from_numpy(xs)
    gate_up = torch.empty((T * 8, 1024), dtype=torch.bfloat16)
    kernels.expert_up_kernel[(T, 8, 1024 // 4)](xq_t, xs_t, w13, s13, ids, gate_up, 4, num_warps=4)
    act_bf16 = kernels.silu_mul(gate_up)
    a, sa = O.silu_mul_quant(gate_up.float().numpy())  # Fish silu_mul_quant restated
    a_t = torch.from_numpy(a).view(torch.float8_e4m3fn)
    sa_t = torch.from_numpy(sa)
    y = torch.empty((T, 2048), dtype=torch.bfloat16)
    kernels.expert_down_kernel[(T, 2048 // 4)](a_t, sa_t, w2, s2, ids, w, y, 4, num_warps=8)
    # atomic down over the same pairs (moe_atomic.py:14-78), block_m 16
    bm = 16
    pairs = T * 8
    max_rows = -(-(pairs + min(pairs, 256) * (bm - 1)) // bm) * bm
    counts = torch.empty(256, dtype=torch.int32)
    starts = torch.empty_like(counts)
    total = torch.empty(1, dtype=torch.int32)
    sorted_ids = torch.full((max_rows,), pairs, dtype=torch.int32)
    expert_ids = torch.zeros((max_rows // bm,), dtype=torch.int32)
    import triton

    kernels.expert_counts_kernel[(256,)](ids, counts, pairs, triton.next_power_of_2(pairs))
    kernels.expert_offsets_kernel[(1,)](counts, starts, total, bm)
    kernels.expert_scatter_kernel[(256,)](
        ids, counts, starts, sorted_ids, expert_ids, pairs, triton.next_power_of_2(pairs),
        triton.next_power_of_2(triton.cdiv(T, bm)), bm)

    class _Ex:
        pass

    ex = _Ex()
    ex.w2_weight, ex.w2_scale_inv = w2, s2
    y_atomic = moe_atomic.atomic_down(a_t, sa_t, ex, w.flatten(), sorted_ids, expert_ids, total, T, bm, 1)
    np.savez_compressed(
        OUT / "small_batch.npz", x=bits(x), router_logits=bits(lgt), ids=ids.numpy(),
        weights=bits(w), experts=sel, wseed_up=np.int64(WSEED_UP), wseed_down=np.int64(WSEED_DOWN),
        xq=xq, xs=xs, gate_up=bits(gate_up), silu_mul=bits(act_bf16), a=a, sa=sa, y=bits(y),
        y_atomic=bits(y_atomic))

    # ---- combine_experts (kernels.py:427-445), gate strided like the packed projection
    T = 5
    routed = bf16(rng.standard_normal((T, 2048)) * 0.3)
    shared = bf16(rng.standard_normal((T, 2048)) * 0.3)
    packed = bf16(rng.standard_normal((T, 1408)) * 2.0)
    gate = packed[:, 1280:1281]
    out = kernels.combine_experts(routed, shared, gate)
    np.savez_compressed(OUT / "combine.npz", routed=bits(routed), shared=bits(shared),
                        gate=bits(gate.contiguous()), out=bits(out))

    # ---- experimental dense FP8: _quantize, _gemv, _gemv_grouped (experimental_fp8.py:10-42)
    N, Kd = 300, 256
    wd = bf16(rng.standard_normal((N, Kd)) * 0.05)
    padded = triton.cdiv(N, 128) * 128
    qf = torch.empty(padded, Kd, dtype=torch.float32)  # register() with an fp32 destination
    sd = torch.empty(padded // 128, Kd // 128, dtype=torch.float32)
    experimental_fp8._quantize[(padded // 128, Kd // 128)](wd, qf, sd, N, Kd, num_warps=8)
    qd = qf.to(torch.float8_e4m3fn)
    experimental_fp8.WEIGHTS[wd.data_ptr()] = (wd, qd, sd)
    xd = bf16(rng.standard_normal((1, Kd)))
    yd = experimental_fp8.linear(xd, wd)
    yg = torch.empty(1, N, dtype=torch.bfloat16)
    experimental_fp8._gemv_grouped[(triton.cdiv(N, 4),)](xd, qd, sd, yg, N, Kd, 4, num_warps=4)
    np.savez_compressed(OUT / "dense_fp8.npz", w=bits(wd), qf32=bits(qf), q=bits(qd), s=bits(sd),
                        x=bits(xd), y=bits(yd), y_grouped=bits(yg))

    # ---- add_norm (kernels.py:405-423): residual update + Gemma RMSNorm
    T = 6
    xa = bf16(rng.standard_normal((T, 2048)) * 0.5)
    res = bf16(rng.standard_normal((T, 2048)) * 2.0)
    res[3] = 0.0  # a row whose update is x itself
    wn = bf16(rng.standard_normal(2048) * 0.1)
    res_in = res.clone()
    on = kernels.add_norm(xa, res, wn, 1e-6)
    np.savez_compressed(OUT / "add_norm.npz", x=bits(xa), residual_in=bits(res_in), weight=bits(wn),
                        residual_out=bits(res), out=bits(on), eps=np.float32(1e-6))
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
