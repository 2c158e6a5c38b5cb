"""Result checks of a GEMM comparison, computed by libemugen on the device.

Mirrors gemm_compare/runner.py:20-55 ``compare_tensors`` and 58-79 ``compare_mse`` (same arguments,
same returned dicts).  The counting pass is one emu_compare kernel; only the per-mismatch samples of
a failing comparison are gathered with torch indexing, on the device.  ``gemm_compare_tensors`` gives
the same dict for an emulated GEMM whose output is never written in full (the comparison fused into
the GEMM's epilogue, emu_gemm_compare).
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


def gemm_compare_tensors(a_fp4: torch.Tensor, b_fp4: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                         real_output: torch.Tensor, *, fmt: int, group_size: int, w_reduce: int,
                         stage3_rounding: int, stage4_rounding: int, alpha: torch.Tensor | None, out_mode: int,
                         sample_count: int = 5) -> dict[str, Any]:
    """``compare_tensors(real_output, emulated GEMM)`` without the emulated [M, N] output in memory: the
    comparison runs in the GEMM's epilogue (emu_gemm_compare: mismatch count, max_diff and the row-major
    index of the first mismatch).  When it finds mismatches, the mismatch samples are those of the
    128-row blocks of A from the first mismatch's block on, recomputed one block at a time (the GEMM of
    a row slice is bit for bit those rows of the whole GEMM) until ``sample_count`` are gathered -- the
    first mismatches in row-major order, as the reference lists them (runner.py:38-49)."""
    from .shard import ROW_BLOCK, row_slice

    kw = dict(fmt=fmt, group_size=group_size, w_reduce=w_reduce, stage3_rounding=stage3_rounding,
              stage4_rounding=stage4_rounding, alpha=alpha, out_mode=out_mode)
    st, _ = _lib.gemm_compare(a_fp4, b_fp4, scale_a, scale_b, real_output, write_out=False, **kw)
    max_diff = float(st["max_diff"])
    status = "SUCCESS" if max_diff == 0 else "MISMATCH"
    details: list[dict[str, Any]] = []
    if status == "MISMATCH" and sample_count > 0:
        M, N = a_fp4.shape[0], b_fp4.shape[0]
        r0 = int(st["first_index"]) // N // ROW_BLOCK * ROW_BLOCK
        while len(details) < sample_count and r0 < M:
            r1 = min(M, r0 + ROW_BLOCK)
            a_rows, sa_rows = row_slice(a_fp4, scale_a, r0, r1)
            rows = _lib.gemm(a_rows, b_fp4, sa_rows, scale_b, **kw)
            sub = compare_tensors(real_output[r0:r1], rows, sample_count=sample_count - len(details))
            for d in sub["mismatch_details"]:
                d["idx"] = (d["idx"][0] + r0, d["idx"][1])
                details.append(d)
            r0 = r1
    return {"status": status, "max_diff": max_diff, "mismatch_details": details}
