"""ctypes binding of libd3moe.so (the C ABI declared in include/d3moe.h).

The library is the only compute path: importing an operator that needs it on a
machine where it is missing raises immediately. There is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("D3MOE_LIB", _HERE / "_lib" / "libd3moe.so"))
# Test-only library (include/d3moe_selftest.h): failure-path probes that the
# product library does not carry.
SELFTEST_LIB_PATH = LIB_PATH.parent / "libd3moe_selftest.so"

D3_OK = 0
D3_EINVAL = -1
D3_ECUDA = -2
D3_EWORKSPACE = -3
D3_EUNSUPPORTED = -4
D3_DTYPE_BF16 = 0
D3_DTYPE_F32 = 1
D3_STATUS_OK = 0
D3_STATUS_WAIT_TIMEOUT = 1
D3_STATUS_BAD_ROW = 2
D3_GATE_UP = 0
D3_UP_GATE = 1
D3_GATE_SWIGLU = 1
D3_GATE_SIGMOID = 2

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_size_t = ctypes.c_size_t


class D3Experts(ctypes.Structure):
    """Mirror of d3_experts_t."""

    _fields_ = [
        ("w13", _c_void_p),
        ("s13", _c_void_p),
        ("w2", _c_void_p),
        ("s2", _c_void_p),
        ("E", _i32),
        ("I", _i32),
        ("H", _i32),
        ("gate_up_order", _i32),
    ]


class D3Rows(ctypes.Structure):
    """Mirror of d3_rows_t (row maps of the mixed decode + prefill call)."""

    _fields_ = [
        ("keep", _c_void_p),
        ("x_rows", _i64),
        ("inverse", _c_void_p),
        ("T_out", _i32),
        ("row_slots", _c_void_p),
        ("row_slots_int64", _i32),
        ("padding_start", _i64),
    ]


# name -> (restype, argtypes); every symbol include/d3moe.h declares.
SIGNATURES: dict[str, tuple] = {
    "d3_version": (_i32, []),
    "d3_last_error_string": (ctypes.c_char_p, []),
    "d3_quant_act_fp8": (_i32, [_c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p, _i32, _c_void_p]),
    "d3_prepare_moe_input": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _i64, _i32, _i32, _i32, _c_void_p, _i32, _i64,
         _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    ),
    "d3_router_logits": (
        _i32, [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _c_void_p, _i64, _c_void_p]
    ),
    "d3_route_topk": (
        _i32,
        [_c_void_p, _i32, _i64, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p],
    ),
    "d3_moe_permute": (
        _i32,
        [_c_void_p, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    ),
    "d3_moe_permute_scratch_size": (_i32, [_i32, ctypes.POINTER(ctypes.c_size_t)]),
    "d3_moe_permute_chunked": (
        _i32,
        [_c_void_p, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    ),
    "d3_silu_mul": (_i32, [_c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p]),
    "d3_silu_mul_quant": (_i32, [_c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p, _c_void_p]),
    "d3_combine_experts": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p]),
    "d3_add_norm": (_i32, [_c_void_p, _c_void_p, _c_void_p, ctypes.c_float, _i32, _i32, _c_void_p, _c_void_p]),
    "d3_combine_experts_add_norm": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _i32, _i32, _c_void_p, _c_void_p,
         ctypes.c_float, _c_void_p, _c_void_p],
    ),
    "d3_fp8_quantize_weight": (_i32, [_c_void_p, _i32, _i32, _c_void_p, _c_void_p, _c_void_p]),
    "d3_fp8_gemv_workspace_size": (_i32, [_i32, _i32, _i32, ctypes.POINTER(_size_t)]),
    "d3_fp8_gemv": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _i64,
         _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
    "d3_fp8_gemv_noalloc": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _i64, _c_void_p],
    ),
    "d3_fp8_gemv_noalloc_status": (_i32, [_c_void_p, _c_void_p]),
    "d3_moe_workspace_size": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_size_t)]),
    "d3_moe_experts": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, ctypes.POINTER(D3Experts),
         ctypes.POINTER(D3Experts), _c_void_p, _c_void_p, _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
    "d3_moe_gate_up_silu": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _i32, _i32, ctypes.POINTER(D3Experts), ctypes.POINTER(D3Experts),
         _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
    "d3_moe_down_combine": (
        _i32,
        [_c_void_p, _i32, _i32, ctypes.POINTER(D3Experts), ctypes.POINTER(D3Experts), _c_void_p,
         _c_void_p, _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
    "d3_set_stage_events": (_i32, [ctypes.POINTER(_c_void_p), _i32]),
    "d3_set_prefill_min_tokens": (_i32, [_i32]),
    "d3_ep_plan_rows": (_i32, [_c_void_p, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p]),
    "d3_route_topk_rows": (
        _i32,
        [_c_void_p, _i32, _i64, _i32, _i32, _i32, _c_void_p, _c_void_p, _i32, _i64, _c_void_p,
         _c_void_p, _i32, _c_void_p],
    ),
    "d3_ep_row_bytes_fp8": (_i32, [_i32, _i32, ctypes.POINTER(_i32)]),
    "d3_ep_pack_fp8": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p,
         _c_void_p],
    ),
    "d3_ep_unpack_fp8": (_i32, [_c_void_p, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "d3_ep_dispatch_meta": (_i32, [_c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p]),
    "d3_combine_pairs": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p],
    ),
    "d3_fp8_gated_gemv": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _i64, _i32, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p,
         _i64, _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
    "d3_moe_experts_fp8": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _i32, _c_void_p, _c_void_p, _i32, _i32,
         ctypes.POINTER(D3Experts), _c_void_p, _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
    "d3_moe_layer": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, ctypes.POINTER(D3Experts),
         ctypes.POINTER(D3Experts), _c_void_p, _c_void_p, _c_void_p, _c_void_p, _size_t,
         _c_void_p, _c_void_p],
    ),
    "d3_moe_layer_add_norm": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, ctypes.POINTER(D3Experts),
         ctypes.POINTER(D3Experts), _c_void_p, _c_void_p, ctypes.c_float, _c_void_p, _c_void_p,
         _c_void_p, _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
    "d3_moe_layer_rows": (
        _i32,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _i32, _i32, ctypes.POINTER(D3Experts),
         ctypes.POINTER(D3Experts), ctypes.POINTER(D3Rows), _c_void_p, _c_void_p, ctypes.c_float,
         _c_void_p, _c_void_p, _c_void_p, _c_void_p, _size_t, _c_void_p, _c_void_p],
    ),
}


class D3Error(RuntimeError):
    """A d3_* entry point returned a negative status."""

    def __init__(self, name: str, code: int, message: str):
        super().__init__(f"{name} failed ({code}): {message}")
        self.code = code


_lib = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load libd3moe.so once and bind every exported symbol."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"libd3moe.so not found at {p}; build it with "
            "`python drama-3-single-b300-inference_b200/build.py` (nvcc, sm_100a)"
        )
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def call(name: str, *args) -> int:
    """Invoke a d3_* entry point and raise D3Error on a negative status.

    Invalid arguments surface as ValueError (the reference raises ValueError
    for shapes/strides, src/drama3/moe_input.py:47-62)."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc < 0:
        msg = (lib.d3_last_error_string() or b"").decode(errors="replace")
        if rc == D3_EINVAL:
            raise ValueError(f"{name}: {msg}")
        raise D3Error(name, rc, msg)
    return rc
