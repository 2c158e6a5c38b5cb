"""Build libemugen.so in-tree: nvcc for sm_100a, C ABI only (no torch headers in the library).

    python -m emugen_b200.build            # -> emugen_b200/libemugen.so
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libemugen.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-fmad=false"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not LIB.is_file():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [REPO / "include" / "emugen.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, *(extra or []), "-I", str(REPO / "include"), "-c", "-o", str(obj), str(src)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    verbose = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else None
    print(build(verbose=verbose, extra=extra))
