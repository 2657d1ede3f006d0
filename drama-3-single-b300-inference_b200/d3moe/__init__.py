"""d3moe — B200-native (sm_100a) FP8 mixture-of-experts hot path of Drama 3.

Drop-in operators with the reference runtime's Python signatures:
  d3moe.kernels          route, small_batch_moe, native_moe, silu_mul,
                         combine_experts, moe_permute
  d3moe.moe_input        prepare_moe_input
  d3moe.experimental_fp8 register, linear (weight-only FP8 dense GEMV)
  d3moe.model            MoEBlock / moe / moe_parts / routed_moe
  d3moe.ep               expert-parallel layer over torch.distributed
All compute runs in libd3moe.so (hand-written CUDA for sm_100a) through the C
ABI of include/d3moe.h; there is no CPU or library fallback.
"""

from . import _lib  # noqa: F401

__all__ = ["_lib"]
