"""Replay of rollout artefacts on the device: the emulated GEMM of every saved case against the real
output saved with it, on one GPU or split over the ranks of a process group.

Artefact format (written by the reference's export harness, gemm_compare/runner.py:299-419 through
gemm_compare/rollout.py:48-79): one ``torch.save`` file holding a dict with
  ``gemm_compare_rollout_version``  1
  ``backend``                       "nvfp" or "mxfp"
  ``seed``, ``meta``                provenance, echoed in the summary
  ``cases``                         a list of dicts, each with ``state`` (the backend's quantised
                                    state dict: gemm_compare/backends/nvfp.py:57-95, mxfp.py:55-94),
                                    ``real_output`` ([M, N] tensor) and ``M``, ``N``, ``K``,
                                    ``dist_a``, ``dist_b`` (``iter`` optional).
``Rollout.read`` checks that shape before any case runs.

Replay (``replay``): rank r of W takes cases r, r + W, ...; every case's verdict goes into one row
of a float64 [cases, 6] table (zeros on the ranks that did not run it) and the table meets in one
``all_reduce(SUM)``, so every rank returns the same code: 0 every case exact (or MSE mode), 1 some
case differs, 2 the artefact's backend is not the requested one (agreed by an all_reduce(MAX)
first).  Without a process group (or with one rank) the same code runs in this process.  The
reference's own ``run_suite_import`` (runner.py:422-526) also runs unchanged with this package's
``emul_fn``; this module adds the device comparison and the split over GPUs.
"""
from __future__ import annotations

import sys
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable

import torch

from .compare import compare_mse, compare_tensors

GemmFn = Callable[[Any], torch.Tensor]
CompareFn = Callable[..., dict]

FORMAT_VERSION = 1
_CASE_KEYS = ("state", "real_output", "M", "N", "K")

# columns of the per-case verdict table exchanged between ranks
_DONE, _MISMATCH, _MAX_DIFF, _MSE_SUM, _MSE_NUMEL, _REF_SQ = range(6)


@dataclass(frozen=True)
class Rollout:
    """A rollout artefact read from disk (tensors on the CPU)."""

    backend: str
    seed: Any
    meta: dict
    cases: list

    @classmethod
    def read(cls, path: str | Path) -> "Rollout":
        """Load and validate an artefact.  Raises ValueError for any other version or a missing field."""
        blob = torch.load(path, map_location="cpu", weights_only=False)
        if not isinstance(blob, dict):
            raise ValueError(f"{path}: not a rollout artefact (a {type(blob).__name__}, not a dict)")
        version = blob.get("gemm_compare_rollout_version")
        if version != FORMAT_VERSION:
            raise ValueError(f"{path}: rollout format version {version!r}, this reader handles {FORMAT_VERSION}")
        backend, cases = blob.get("backend"), blob.get("cases")
        if not isinstance(backend, str) or not isinstance(cases, list):
            raise ValueError(f"{path}: rollout artefact without a backend name or a case list")
        for i, case in enumerate(cases):
            missing = [k for k in _CASE_KEYS if k not in case]
            if missing:
                raise ValueError(f"{path}: case {i} lacks {', '.join(missing)}")
        return cls(backend.lower(), blob.get("seed"), dict(blob.get("meta") or {}), cases)

    def state(self, i: int, device: str | torch.device):
        """The quantised state of case i, rebuilt by its backend's deserialiser on `device`."""
        if self.backend == "nvfp":
            from .backends.nvfp import nvfp_quant_state_from_dict as from_dict
        elif self.backend == "mxfp":
            from .backends.mxfp import mxfp_quant_state_from_dict as from_dict
        else:
            raise ValueError(f"rollout backend {self.backend!r} is neither 'nvfp' nor 'mxfp'")
        return from_dict(self.cases[i]["state"], device=device)


def _verdict_row(case: dict, state, emul_fn: GemmFn, device, metric_mode: str, sample_count: int,
                 cmp_exact: CompareFn, cmp_mse: CompareFn) -> tuple[torch.Tensor, dict]:
    real = case["real_output"].to(device)
    emulated = emul_fn(state)
    row = torch.zeros(6, dtype=torch.float64)
    row[_DONE] = 1.0
    if metric_mode == "exact":
        c = cmp_exact(real, emulated, sample_count=sample_count)
        row[_MISMATCH] = 1.0 if c["status"] == "MISMATCH" else 0.0
        row[_MAX_DIFF] = float(c["max_diff"])
    elif metric_mode == "mse":
        c = cmp_mse(real, emulated)
        row[_MSE_SUM], row[_MSE_NUMEL] = float(c["mse_sum"]), float(c["mse_numel"])
        row[_REF_SQ], row[_MAX_DIFF] = float(c["real_sq_sum"]), float(c["max_mse"])
    else:
        raise ValueError(f"unknown metric_mode={metric_mode!r}")
    return row, c


def _report(title: str, rollout: Rollout, table: torch.Tensor, metric_mode: str) -> None:
    done = table[:, _DONE] > 0
    n, ran = table.shape[0], int(done.sum())
    print(f"{title}: {ran}/{n} cases replayed (backend {rollout.backend}, artefact seed {rollout.seed})")
    if metric_mode == "mse":
        numel = float(table[done, _MSE_NUMEL].sum())
        rel = [float(s) ** 0.5 / max(float(r) ** 0.5, 1e-12) for s, r in zip(table[done, _MSE_SUM], table[done, _REF_SQ])]
        print(f"  MSE {float(table[done, _MSE_SUM].sum()) / max(numel, 1.0):.8e}, "
              f"mean relative L2 error {sum(rel) / max(len(rel), 1):.8e}, "
              f"worst element {float(table[done, _MAX_DIFF].max()) if ran else 0.0:.8e}")
        return
    bad = [i for i in range(n) if done[i] and table[i, _MISMATCH] > 0]
    print(f"  bit-exact: {ran - len(bad)}, differing: {len(bad)}" +
          (f" (cases {bad[:20]}{' ...' if len(bad) > 20 else ''})" if bad else ""))


def replay(emul_fn: GemmFn, *, backend: str, artifact_path: str | Path, device: str = "cuda",
           metric_mode: str = "exact", sample_count: int = 5, compare_fn: CompareFn = compare_tensors,
           mse_fn: CompareFn = compare_mse, group=None, distributed: bool = True,
           title: str = "rollout replay") -> int:
    """Replay an artefact with `emul_fn`, split over `group`'s ranks when `distributed` and a process
    group is initialised (every rank must then call this), else in this process alone.  Returns
    0 / 1 / 2 (module doc)."""
    import torch.distributed as dist

    split = distributed and dist.is_available() and dist.is_initialized()
    rank, world = (dist.get_rank(group), dist.get_world_size(group)) if split else (0, 1)
    try:
        rollout = Rollout.read(artifact_path)
        wrong_backend = rollout.backend != backend.lower()
    except (OSError, ValueError) as e:
        print(f"[rank {rank}] cannot replay {artifact_path}: {e}", file=sys.stderr)
        rollout, wrong_backend = None, True
    comm = (torch.device("cuda", torch.cuda.current_device())
            if split and dist.get_backend(group) == "nccl" else torch.device("cpu"))
    if split:
        flag = torch.tensor([1.0 if wrong_backend else 0.0], dtype=torch.float64, device=comm)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)   # one verdict for all ranks
        wrong_backend = bool(flag.item() > 0)
    if wrong_backend:
        if rank == 0 and rollout is not None:
            print(f"ERROR: artifact backend {rollout.backend!r} != requested backend {backend.lower()!r}",
                  file=sys.stderr)
        return 2
    table = torch.zeros((len(rollout.cases), 6), dtype=torch.float64)
    for i in range(rank, len(rollout.cases), world):
        try:
            table[i], _ = _verdict_row(rollout.cases[i], rollout.state(i, device), emul_fn, device, metric_mode,
                                       sample_count, compare_fn, mse_fn)
        except Exception as e:  # reported per case; the case stays out of the verdict
            print(f"[rank {rank}] case {i}: {type(e).__name__}: {e}", file=sys.stderr)
    if split:
        t = table.to(comm)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        table = t.cpu()
    if rank == 0:
        _report(title, rollout, table, metric_mode)
    if metric_mode == "mse":
        return 0
    return 1 if bool((table[:, _MISMATCH] > 0).any()) else 0


def run_suite_import(emul_fn: GemmFn, *, backend: str, artifact_path: str | Path, device: str = "cuda",
                     sample_count: int = 5, metric_mode: str = "exact", compare_fn: CompareFn = compare_tensors,
                     mse_fn: CompareFn = compare_mse, **_ignored) -> int:
    """Single-process replay with the arguments and return codes of the reference's
    ``run_suite_import`` (gemm_compare/runner.py:422-433); printing options are accepted and ignored."""
    return replay(emul_fn, backend=backend, artifact_path=artifact_path, device=device, sample_count=sample_count,
                  metric_mode=metric_mode, compare_fn=compare_fn, mse_fn=mse_fn, distributed=False)


def run_suite_import_sharded(emul_fn: GemmFn, *, backend: str, artifact_path: str | Path, device: str = "cuda",
                             sample_count: int = 5, metric_mode: str = "exact", compare_fn: CompareFn = compare_tensors,
                             mse_fn: CompareFn = compare_mse, group=None, **_ignored) -> int:
    """``replay`` over the ranks of the default (or given) process group."""
    return replay(emul_fn, backend=backend, artifact_path=artifact_path, device=device, metric_mode=metric_mode,
                  sample_count=sample_count, compare_fn=compare_fn, mse_fn=mse_fn, group=group,
                  title="rollout replay (sharded)")

