"""Builds libd3moe.so (every CUDA source under csrc/) for sm_100a with nvcc.

The library is written in-tree next to the Python package
(d3moe/_lib/libd3moe.so) so that it travels with the source tree; it is
rebuilt only when a source or header is newer than the library.

Usage: python build.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT_DIR = HERE / "d3moe" / "_lib"
LIB = OUT_DIR / "libd3moe.so"
# test-only library (csrc/selftest/): failure-path probes kept out of the product
SELFTEST_LIB = OUT_DIR / "libd3moe_selftest.so"
INCLUDE = HERE.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libd3moe.so")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not LIB.exists() or not SELFTEST_LIB.exists():
        return True
    lib_time = min(LIB.stat().st_mtime, SELFTEST_LIB.stat().st_mtime)
    deps = list(CSRC.rglob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > lib_time for p in deps if p.is_file())


def _link(cc: str, srcs: list[Path], out: Path, objdir: Path, verbose: bool) -> None:
    objs = []
    for src in srcs:
        obj = objdir / (src.stem + ".o")
        cmd = [cc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = out.with_suffix(".so.tmp")
    cmd = [cc, *ARCH_FLAGS, "-shared", "-Xlinker", "--no-undefined", "-o", str(tmp), *objs, "-lcudart"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    cc = nvcc()
    _link(cc, sources(), LIB, objdir, verbose)
    _link(cc, sorted((CSRC / "selftest").glob("*.cu")), SELFTEST_LIB, objdir, verbose)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
