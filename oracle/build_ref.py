"""Compile the reference's own C++ emulators, unmodified, from where they lie in the reference tree.

Outputs go only to ``oracle/_ref/`` (git-ignored; it travels with the repository snapshot so the
benchmark's CPU-baseline leg can time the reference on the GPU host).  This is the same JIT
recipe the reference uses (``torch.utils.cpp_extension.load`` of one ``.cpp``,
``nvfp_cpp_emul/nvfp_cpp_emul/__init__.py:46-66``), with the build directory pointed here.

Test infrastructure only: nothing in the product path imports what this builds.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

SOURCES = {
    "nvfp": ("nvfp_emul_jit", "nvfp_cpp_emul/nvfp_cpp_emul/csrc/nvfp_emulation.cpp"),
    "mxfp": ("mxfp_emul_jit", "mxfp_cpp_emul/mxfp_cpp_emul/csrc/mxfp_emulation.cpp"),
}


def build(reference: Path, out: Path, verbose: bool = False) -> dict[str, Path]:
    from torch.utils.cpp_extension import load

    built = {}
    for key, (name, rel) in SOURCES.items():
        src = reference / rel
        if not src.is_file():
            raise FileNotFoundError(src)
        bdir = out / key
        bdir.mkdir(parents=True, exist_ok=True)
        load(name=name, sources=[str(src)], build_directory=str(bdir), verbose=verbose)
        built[key] = bdir / f"{name}.so"
    return built


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EMUGEN_REFERENCE"),
                    help="root of the reference source tree (default: $EMUGEN_REFERENCE)")
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent / "_ref"))
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set EMUGEN_REFERENCE")
    ref = Path(args.reference)
    if not ref.is_dir():
        print(f"reference tree not present at {ref}; nothing to build", file=sys.stderr)
        return 0
    for k, p in build(ref, Path(args.out), args.verbose).items():
        print(k, p, os.path.getsize(p))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
