"""Result checks of a GEMM comparison, computed by libemugen on the device.

Mirrors gemm_compare/runner.py:20-55 ``compare_tensors`` and 58-79 ``compare_mse`` (same arguments,
same returned dicts).  The counting pass is one emu_compare kernel; only the per-mismatch samples of
a failing comparison are gathered with torch indexing, on the device.
"""
from __future__ import annotations

from typing import Any

import torch

from . import _lib


def compare_tensors(real_output: torch.Tensor, modeling_res: torch.Tensor, *, sample_count: int = 5
                    ) -> dict[str, Any]:
    """Exact match with NaN agreement: an element mismatches when it is neither == (+0 == -0) nor
    NaN on both sides.  max_diff is max |real - model| over mismatches (NaN differences -> inf)."""
    st = _lib.compare_stats(real_output, modeling_res)
    max_diff = float(st["max_diff"])
    status = "SUCCESS" if max_diff == 0 else "MISMATCH"
    details: list[dict[str, Any]] = []
    if status == "MISMATCH" and sample_count > 0:
        dev = real_output.device if real_output.is_cuda else modeling_res.device
        r = real_output.to(dev)
        m = modeling_res.to(dev)
        bad = ~((r == m) | (r.isnan() & m.isnan()))
        for row in torch.nonzero(bad, as_tuple=False)[:sample_count].tolist():
            pos = tuple(row)
            rv, mv = r[pos], m[pos]
            d = (rv.float() - mv.float()).abs()
            details.append({"idx": pos, "real": rv.item(), "model": mv.item(),
                            "diff": float("inf") if bool(torch.isnan(d)) else d.item()})
    return {"status": status, "max_diff": max_diff, "mismatch_details": details}


def compare_mse(reference: torch.Tensor, target: torch.Tensor) -> dict[str, Any]:
    """Squared-error statistics with non-finite terms dropped, plus ||reference||^2 for the
    relative L2 error (sums in f64 on the device; the reference sums in f32)."""
    st = _lib.compare_stats(reference, target)
    sq_sum = float(st["sq_error_sum"])
    ref_sq_sum = float(st["ref_sq_sum"])
    numel = int(st["numel"])
    return {
        "status": "OK",
        "mean_mse": sq_sum / max(numel, 1),
        "max_mse": float(st["max_sq_error"]),
        "mse_sum": sq_sum,
        "mse_numel": numel,
        "real_sq_sum": ref_sq_sum,
        "per_gemm_rel_l2_error": (sq_sum ** 0.5) / max(ref_sq_sum ** 0.5, 1e-12),
        "mismatch_details": [],
    }
