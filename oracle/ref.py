"""Load the reference's own C++ emulators compiled by ``build_ref.py`` into ``oracle/_ref``.

TEST INFRASTRUCTURE / CPU BASELINE ONLY.  Returns None when they were not built (e.g. the
reference tree was never mounted where the build ran).
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
from pathlib import Path

HERE = Path(__file__).resolve().parent
_cache: dict[str, object] = {}


def load(kind: str):
    """kind: 'nvfp' -> module with emulated_scaled_fp4_mm; 'mxfp' -> emulated_mxfp4_mm."""
    if kind in _cache:
        return _cache[kind]
    import torch  # noqa: F401  (libtorch symbols must be loaded first)

    name = {"nvfp": "nvfp_emul_jit", "mxfp": "mxfp_emul_jit"}[kind]
    so = HERE / "_ref" / kind / f"{name}.so"
    if not so.is_file():
        _cache[kind] = None
        return None
    loader = importlib.machinery.ExtensionFileLoader(name, str(so))
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    _cache[kind] = mod
    return mod
