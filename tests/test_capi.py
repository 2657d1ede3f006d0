"""CPU checks of the drop-in boundary: libd3moe.so loads, exports every entry
point include/d3moe.h declares, and its host-side argument checks behave
(no kernel is launched in these tests)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "d3moe.h"
LIB = ROOT / "drama-3-single-b300-inference_b200" / "d3moe" / "_lib" / "libd3moe.so"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"D3_API\s+[\w\s\*]+?\b(d3_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        import subprocess
        import sys
        subprocess.run([sys.executable, str(LIB.parents[2] / "build.py")], check=True)
    from d3moe import _lib
    return _lib.load()


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for name in ("d3_route_topk", "d3_moe_permute", "d3_moe_experts", "d3_moe_layer", "d3_fp8_gemv",
                 "d3_prepare_moe_input", "d3_router_logits", "d3_combine_experts", "d3_silu_mul"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    from d3moe import _lib
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in d3moe.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_selftest_library_is_separate_and_exports_its_probe(lib):
    """The failure-path probe ships in the test-only libd3moe_selftest.so
    (include/d3moe_selftest.h), not in the product library."""
    from d3moe import _lib
    text = (ROOT / "include" / "d3moe_selftest.h").read_text()
    syms = sorted(set(re.findall(r"D3_API\s+[\w\s\*]+?\b(d3_\w+)\s*\(", text)))
    assert syms == ["d3_wait_timeout_probe"]
    st = ctypes.CDLL(str(_lib.SELFTEST_LIB_PATH))
    for name in syms:
        assert hasattr(st, name)
        assert not hasattr(lib, name), f"{name} leaked into the product library"


def test_version_and_error_string(lib):
    assert lib.d3_version() >= 1
    assert isinstance(lib.d3_last_error_string(), bytes)


def test_workspace_sizes_are_host_only(lib):
    from d3moe import _lib
    n = ctypes.c_size_t()
    assert lib.d3_moe_workspace_size(64, 8, 128, 768, 2048, 1, ctypes.byref(n)) == 0
    P, R = 64 * 8, 64 * 9
    # activation rows, requantised rows and fp32 expert rows dominate
    assert n.value >= R * 2048 + R * 768 + R * 2048 * 4
    assert lib.d3_moe_workspace_size(0, 8, 128, 768, 2048, 1, ctypes.byref(n)) == 0
    assert lib.d3_moe_workspace_size(-1, 8, 128, 768, 2048, 1, ctypes.byref(n)) == _lib.D3_EINVAL
    assert lib.d3_fp8_gemv_workspace_size(64, 4096, 2048, ctypes.byref(n)) == 0
    assert n.value >= 64 * 2048 * 2
    assert lib.d3_fp8_gemv_workspace_size(64, 4096, 100, ctypes.byref(n)) == _lib.D3_EINVAL


def test_invalid_arguments_fail_before_launch(lib):
    from d3moe import _lib
    # H not a multiple of 128
    rc = lib.d3_quant_act_fp8(None, 100, 4, 100, None, None, 0, None)
    assert rc == _lib.D3_EINVAL
    assert b"multiple of 128" in lib.d3_last_error_string()
    # k larger than E
    rc = lib.d3_route_topk(None, 0, 4, 4, 4, 8, None, None, None, 0, None)
    assert rc == _lib.D3_EINVAL
    # permute with too small a destination
    rc = lib.d3_moe_permute(None, 64, 8, 128, 16, None, None, None, None, None, 16, None, None,
                            None, None)
    assert rc == _lib.D3_EINVAL
    # experts struct with bad geometry
    ex = _lib.D3Experts(16, 16, 16, 16, 128, 700, 2048)
    rc = lib.d3_moe_experts(16, 2048, None, None, 4, 8, ctypes.byref(ex), None, None, None, None, 0,
                            None, None)
    assert rc == _lib.D3_EINVAL
    assert b"multiples of 128" in lib.d3_last_error_string()


def test_expert_parallel_entry_points_check_arguments(lib):
    from d3moe import _lib
    n = ctypes.c_int(0)
    assert lib.d3_ep_row_bytes_fp8(2048, 8, ctypes.byref(n)) == _lib.D3_OK
    assert n.value == 2192 and n.value % 16 == 0
    assert lib.d3_ep_row_bytes_fp8(2000, 8, ctypes.byref(n)) == _lib.D3_EINVAL
    # more ranks than the planner supports
    rc = lib.d3_ep_plan_rows(ctypes.c_void_p(16), 4, 8, 16, 4096, ctypes.c_void_p(16),
                             ctypes.c_void_p(16), None)
    assert rc == _lib.D3_EINVAL
    # pack: H not a multiple of 128
    rc = lib.d3_ep_pack_fp8(ctypes.c_void_p(256), 100, ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 8,
                            100, 16, 2, None, ctypes.c_void_p(256), None)
    assert rc == _lib.D3_EINVAL
    # unpack: received rows not 16-byte aligned
    rc = lib.d3_ep_unpack_fp8(ctypes.c_void_p(264), 4, 8, 2048, ctypes.c_void_p(256),
                              ctypes.c_void_p(256), ctypes.c_void_p(256), None)
    assert rc == _lib.D3_EINVAL
    assert b"16-byte aligned" in lib.d3_last_error_string()


def test_down_stage_refuses_an_unfilled_workspace(lib):
    """d3_moe_down_combine checks its host-side record of the first stage
    before anything reaches the device."""
    from d3moe import _lib
    ex = _lib.D3Experts(16, 16, 16, 16, 128, 768, 2048)
    need = ctypes.c_size_t()
    assert lib.d3_moe_workspace_size(4, 8, 128, 768, 2048, 0, ctypes.byref(need)) == 0
    rc = lib.d3_moe_down_combine(16, 4, 8, ctypes.byref(ex), None, 256, None, 4096, need.value,
                                 None, None)
    assert rc == _lib.D3_EINVAL
    assert b"not filled by d3_moe_gate_up_silu" in lib.d3_last_error_string()


def test_python_wrappers_reject_cpu_tensors():
    torch = pytest.importorskip("torch")
    from d3moe import kernels, moe_input
    x = torch.zeros(4, 2048, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        kernels.route(torch.zeros(4, 128, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        moe_input.prepare_moe_input(x, torch.zeros(4, 256, dtype=torch.bfloat16))


def test_prepare_moe_input_reference_errors():
    torch = pytest.importorskip("torch")
    from d3moe import moe_input
    x = torch.zeros(4, 2048, dtype=torch.bfloat16)
    r = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="Channel strides"):
        moe_input.prepare_moe_input(x.t().contiguous().t(), r)
    with pytest.raises(ValueError, match="both row_slots"):
        moe_input.prepare_moe_input(x, r, row_slots=torch.zeros(4, dtype=torch.int64))
    with pytest.raises(ValueError, match="padding_start"):
        moe_input.prepare_moe_input(x, r, row_slots=torch.zeros(4, dtype=torch.int64), padding_start=0)
