"""Loader for the committed golden fixtures (tests/golden/emul_golden.npz + manifest.json)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_cases():
    man = json.loads((GOLDEN / "manifest.json").read_text())
    data = np.load(GOLDEN / "emul_golden.npz")
    out = []
    for i, c in enumerate(man["cases"]):
        c = dict(c)
        c["id"] = i
        for k in ("a", "b", "sfa", "sfb", "out"):
            c[k] = data[f"c{i}_{k}"]
        out.append(c)
    return out


def nan_equal_mismatches(x_bits: np.ndarray, y_bits: np.ndarray, dtype: str) -> int:
    """Count elements that differ bitwise, treating any NaN as equal to any NaN (the reference's
    ``compare_tensors`` rule, gemm_compare/runner.py:20-32, minus its +0 == -0 leniency)."""
    x = x_bits.astype(np.uint16)
    y = y_bits.astype(np.uint16)
    if dtype == "float16":
        isnan = lambda b: ((b & 0x7C00) == 0x7C00) & ((b & 0x03FF) != 0)
    else:
        isnan = lambda b: ((b & 0x7F80) == 0x7F80) & ((b & 0x007F) != 0)
    eq = (x == y) | (isnan(x) & isnan(y))
    return int((~eq).sum())
