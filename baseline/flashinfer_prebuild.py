"""Prebuilds FlashInfer's trtllm fused-MoE launcher module for sm_100a into
baseline/_flashinfer/ (git-ignored), so that bench.py can time the
reference's own Blackwell MoE kernel (trtllm_fp8_block_scale_moe, called by
src/drama3/model.py:556-580) on a GPU box without compiling it there.

FlashInfer JIT-compiles this launcher (host code around its closed trtllm-gen
cubins, which ship in the flashinfer-cubin wheel) on first use; that takes
tens of minutes of nvcc time. Run this once on any machine with nvcc:

    python baseline/flashinfer_prebuild.py

The result is copied to baseline/_flashinfer/aot/<module>/<module>.so, where
bench.py points FlashInfer's prebuilt-module directory. Nothing here is part
of the product library.
"""

from __future__ import annotations

import os
import shutil
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_flashinfer"


def main() -> int:
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ["FLASHINFER_WORKSPACE_BASE"] = str(OUT)
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")
    t0 = time.time()
    from flashinfer.jit.fused_moe import gen_trtllm_gen_fused_moe_sm100_module

    spec = gen_trtllm_gen_fused_moe_sm100_module()
    spec.build(verbose=False)
    lib = spec.jit_library_path
    dst = OUT / "aot" / spec.name / f"{spec.name}.so"
    dst.parent.mkdir(parents=True, exist_ok=True)
    shutil.copy2(lib, dst)
    print(f"{dst} ({time.time() - t0:.0f} s)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
