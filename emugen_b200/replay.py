"""Replay of rollout artefacts: the emulated GEMM of every saved case against its saved real output.

``run_suite_import`` mirrors gemm_compare/runner.py:422-526 (same arguments, printout and return
code: 0 all exact / MSE mode, 1 mismatches, 2 backend mismatch) with the comparison done on the
device (``emugen_b200.compare``).  ``run_suite_import_sharded`` runs the same replay on every rank of
an initialised ``torch.distributed`` process group: rank r takes cases r, r + world, ...; the per-case
results travel in one ``all_reduce(SUM)`` of a float64 [cases, 6] tensor (a case is filled in by
exactly one rank, zeros elsewhere), and every rank returns the same code; rank 0 prints.
"""
from __future__ import annotations

import sys
import traceback
from pathlib import Path
from typing import Any, Callable

import torch

from .compare import compare_mse, compare_tensors
from .rollout import load_rollout_artifact, quant_state_from_dict

GemmFn = Callable[[Any], torch.Tensor]
CompareFn = Callable[..., dict]

# columns of the per-case result rows exchanged between ranks
_DONE, _MISMATCH, _MAX_DIFF, _MSE_SUM, _MSE_NUMEL, _REF_SQ = range(6)


def _replay_case(row: dict[str, Any], idx: int, emul_fn: GemmFn, backend: str, device: str, metric_mode: str,
                 sample_count: int, cmp_exact: CompareFn, cmp_mse: CompareFn) -> dict[str, Any]:
    state = quant_state_from_dict(row["state"], backend, device=device)
    real_output = row["real_output"].to(device)
    modeling_res = emul_fn(state)
    if metric_mode == "exact":
        cmp = cmp_exact(real_output, modeling_res, sample_count=sample_count)
    elif metric_mode == "mse":
        cmp = cmp_mse(real_output, modeling_res)
    else:
        raise ValueError(f"unknown metric_mode={metric_mode!r}")
    return {"iter": row.get("iter", idx), "M": row["M"], "N": row["N"], "K": row["K"], "dist_a": row["dist_a"],
            "dist_b": row["dist_b"], **cmp}


def _summary(name: str, n_cases: int, results: list[dict[str, Any]], metric_mode: str) -> int:
    print("\n" + "=" * 70)
    print(f"SUMMARY | {name}")
    print("=" * 70)
    if metric_mode == "mse":
        total_numel = sum(int(r.get("mse_numel", 0)) for r in results)
        total_mse_sum = sum(float(r.get("mse_sum", 0.0)) for r in results)
        mean_mse = total_mse_sum / max(total_numel, 1)
        per_gemm = [float(r.get("per_gemm_rel_l2_error", 0.0)) for r in results]
        mean_per_gemm = sum(per_gemm) / max(len(per_gemm), 1)
        worst = max((float(r.get("max_mse", 0.0)) for r in results), default=0.0)
        print(f"Total: {n_cases}, Completed: {len(results)}")
        print(f"MSE mean: {mean_mse:.8e}")
        print(f"mean over GEMMs of sqrt(sum(error^2)) / sqrt(sum(real^2)): {mean_per_gemm:.8e}")
        print(f"MSE max (worst element): {worst:.8e}")
        return 0
    mismatches = [r for r in results if r["status"] == "MISMATCH"]
    print(f"Total: {n_cases}, Matches: {len(results) - len(mismatches)}, Mismatches: {len(mismatches)}")
    print("=" * 70)
    if not mismatches:
        print("*** All tests: exact bitwise match ***")
        return 0
    print(f"Exact-match rate: {(len(results) - len(mismatches)) / max(len(results), 1) * 100:.2f}%")
    return 1


def _load_checked(artifact_path, backend: str):
    data = load_rollout_artifact(artifact_path, map_location="cpu")
    art_backend = str(data["backend"]).lower()
    if art_backend != backend.lower():
        print(f"ERROR: artifact backend {art_backend!r} != CLI backend {backend.lower()!r}", file=sys.stderr)
        return None
    return data


def run_suite_import(emul_fn: GemmFn, *, backend: str, artifact_path: str | Path, name: str = "GEMM compare import",
                     device: str = "cuda", sample_count: int = 5, max_mismatch_print: int = 20,
                     metric_mode: str = "exact", print_iter_status: bool = True,
                     compare_fn: CompareFn = compare_tensors, mse_fn: CompareFn = compare_mse) -> int:
    """Replay a saved rollout on this device and compare with the saved real outputs."""
    data = _load_checked(artifact_path, backend)
    if data is None:
        return 2
    cases: list[dict[str, Any]] = list(data["cases"])
    print(f"\n{'=' * 70}\n{name}\n{'=' * 70}")
    print(f"Mode: IMPORT <- {artifact_path}")
    print(f"artifact seed = {data.get('seed')}")
    print(f"artifact meta = {data.get('meta', {})}")
    print(f"Cases: {len(cases)} | device = {device}")
    print("=" * 70)
    results: list[dict[str, Any]] = []
    printed = 0
    for idx, row in enumerate(cases):
        print(f"\rImport {idx + 1}/{len(cases)}: iter={row.get('iter')} ... ", end="")
        sys.stdout.flush()
        try:
            out = _replay_case(row, idx, emul_fn, backend, device, metric_mode, sample_count, compare_fn, mse_fn)
            results.append(out)
            print(out["status"] if print_iter_status else "OK")
            if metric_mode == "exact" and out["status"] == "MISMATCH" and printed < max_mismatch_print:
                printed += 1
                print("    >>> Mismatch Details:")
                for d in out["mismatch_details"]:
                    print(f"      Pos {d['idx']}: Real={d['real']:.6f} | Model={d['model']:.6f} | Diff={d['diff']:.6f}")
        except Exception as e:  # reported per case, as the reference does
            print(f"\nFATAL ERROR on import case {idx + 1}: {e}")
            traceback.print_exc()
    return _summary(name, len(cases), results, metric_mode)


def run_suite_import_sharded(emul_fn: GemmFn, *, backend: str, artifact_path: str | Path,
                             name: str = "GEMM compare import (sharded)", device: str = "cuda",
                             sample_count: int = 5, metric_mode: str = "exact",
                             compare_fn: CompareFn = compare_tensors, mse_fn: CompareFn = compare_mse,
                             group=None) -> int:
    """run_suite_import over all ranks of the default (or given) process group."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    data = _load_checked(artifact_path, backend)
    bad_backend = torch.tensor([0.0 if data is not None else 1.0], dtype=torch.float64)
    cases: list[dict[str, Any]] = list(data["cases"]) if data is not None else []
    n = torch.tensor([float(len(cases))], dtype=torch.float64)
    comm_dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    head = torch.cat([bad_backend, n]).to(comm_dev)
    dist.all_reduce(head, op=dist.ReduceOp.MAX, group=group)   # every rank sees the same verdict
    if head[0].item() > 0:
        return 2
    table = torch.zeros((len(cases), 6), dtype=torch.float64)
    for idx in range(rank, len(cases), world):
        row = cases[idx]
        try:
            out = _replay_case(row, idx, emul_fn, backend, device, metric_mode, sample_count, compare_fn, mse_fn)
        except Exception as e:
            print(f"[rank {rank}] FATAL ERROR on import case {idx + 1}: {e}", file=sys.stderr)
            continue
        table[idx, _DONE] = 1.0
        if metric_mode == "exact":
            table[idx, _MISMATCH] = 1.0 if out["status"] == "MISMATCH" else 0.0
            table[idx, _MAX_DIFF] = float(out["max_diff"])
        else:
            table[idx, _MSE_SUM] = float(out["mse_sum"])
            table[idx, _MSE_NUMEL] = float(out["mse_numel"])
            table[idx, _REF_SQ] = float(out["real_sq_sum"])
            table[idx, _MAX_DIFF] = float(out["max_mse"])
    t = table.to(comm_dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    table = t.cpu()
    results: list[dict[str, Any]] = []
    for idx in range(len(cases)):
        if table[idx, _DONE] == 0:
            continue
        if metric_mode == "exact":
            results.append({"status": "MISMATCH" if table[idx, _MISMATCH] > 0 else "SUCCESS",
                            "max_diff": float(table[idx, _MAX_DIFF])})
        else:
            s, ne, rs = (float(table[idx, c]) for c in (_MSE_SUM, _MSE_NUMEL, _REF_SQ))
            results.append({"status": "OK", "mse_sum": s, "mse_numel": int(ne), "real_sq_sum": rs,
                            "max_mse": float(table[idx, _MAX_DIFF]),
                            "per_gemm_rel_l2_error": (s ** 0.5) / max(rs ** 0.5, 1e-12)})
    if rank == 0:
        return _summary(name, len(cases), results, metric_mode)
    if metric_mode == "mse":
        return 0
    return 1 if any(r["status"] == "MISMATCH" for r in results) else 0
