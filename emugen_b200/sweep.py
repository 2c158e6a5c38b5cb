"""Accumulator-model sweeps: one quantised GEMM case evaluated under many accumulator models (alignment
widths, aligned-addend rounding, accumulate size, summation order) and compared with a reference
output, on the device.  The reference runs such sweeps one model at a time from its search scripts
(search/w3.py:123-158, search/w4.py:60-90), each a host loop over the libtorch emulation; its
MMAEngine accepts the width parameters without using them (search/emulation/core.py:31-38), so the
models here have no reference counterpart (see emulation.AccumModel).

``run_sweep`` evaluates every model on the caller's device: models whose block size is 1, 2, 4 or 8
groups go through ``emu_gemm_sweep`` (stages 1-2 once per group for all models of a block size, each
model compared with the reference inside the kernel), others one at a time through emu_gemm_model and
the device comparison.  ``run_sweep_sharded`` splits the models
over the ranks of a process group: rank 0's quantised case and reference output are broadcast once,
rank r evaluates models r, r + world, ..., and the per-model results meet in one all_reduce(SUM)
of an int64 [models, 2] table (mismatch count, evaluated flag), so every rank returns the same
table.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch

from . import _lib
from .emulation import AccumModel, _rounding_code


@dataclass(frozen=True)
class SweepConfig:
    """One point of a sweep: the accumulator model plus the block size and stage-4 rounding it runs with."""

    model: AccumModel
    w_reduce: int
    stage4_rounding: int = _lib.EMU_RZ


@dataclass
class SweepCase:
    """A quantised GEMM case: packed operands, swizzled block scales, format, alpha (NVFP4) or None."""

    a_fp4: torch.Tensor
    b_fp4: torch.Tensor
    scale_a: torch.Tensor
    scale_b: torch.Tensor
    fmt: int                      # _lib.EMU_FMT_NVFP4 / EMU_FMT_MXFP4
    alpha: Optional[torch.Tensor] = None

    @property
    def group_size(self) -> int:
        return 16 if self.fmt == _lib.EMU_FMT_NVFP4 else 32


def default_configs() -> list[SweepConfig]:
    """The MXFP4 sweep of the benchmark configuration: alignment width 24..31 at both stages x {RZ, RNE}
    alignment rounding x accumulate size {32, 64, 128} (w_reduce 1, 2, 4), then 8 summation orders
    (reverse and pairwise x w_reduce {2, 4} x stage-4 {RZ, RNE}) -- 56 configurations.

    Accumulate size 16 is not in the grid because it is undefined for MXFP4: the emulation sums whole
    scale groups (one fp16-rounded dot product per group, then w_reduce groups per stage-3 block,
    search/emulation/core.py:57-66, 95-101), and an MXFP4 group is 32 elements, so the smallest
    accumulation is one group (w_reduce 1 = 32 elements).  For NVFP4 (16-element groups) accumulate
    size 16 is w_reduce 1."""
    from .emulation import RoundStrategy

    cfgs = [SweepConfig(AccumModel(align3=w, align4=w, align_rounding=rm), wr)
            for w in range(24, 32) for rm in (RoundStrategy.RZ, RoundStrategy.RNE) for wr in (1, 2, 4)]
    cfgs += [SweepConfig(AccumModel(order=o), wr, r4)
             for o in (1, 2) for wr in (2, 4) for r4 in (_lib.EMU_RZ, _lib.EMU_RNE)]
    return cfgs


def evaluate(case: SweepCase, cfg: SweepConfig, reference: torch.Tensor) -> int:
    """Mismatch count of one model against `reference` (bf16: the model's f32 result is rounded to
    bf16 once, as a hardware epilogue rounds; f16 / f32 references compare in their own type)."""
    out_mode = _lib.EMU_OUT_F32
    out = _lib.gemm_model(case.a_fp4, case.b_fp4, case.scale_a, case.scale_b, fmt=case.fmt,
                          group_size=case.group_size, w_reduce=cfg.w_reduce, stage3_rounding=_lib.EMU_RZ,
                          stage4_rounding=cfg.stage4_rounding, alpha=case.alpha, out_mode=out_mode,
                          align3=cfg.model.align3, align4=cfg.model.align4,
                          align_rounding=_rounding_code(cfg.model.align_rounding), order=cfg.model.order)
    return int(_lib.compare_stats(reference, out.to(reference.dtype))["mismatches"])


BATCH_W_REDUCE = (1, 2, 4, 8)


def evaluate_batch(case: SweepCase, configs: Sequence[SweepConfig], reference: torch.Tensor) -> list[int]:
    """Mismatch counts of several models in one emu_gemm_sweep call (block sizes in BATCH_W_REDUCE),
    the same counts evaluate() gives model by model."""
    models = [(c.w_reduce, c.stage4_rounding, c.model.align3, c.model.align4,
               _rounding_code(c.model.align_rounding), c.model.order) for c in configs]
    return _lib.gemm_sweep(case.a_fp4, case.b_fp4, case.scale_a, case.scale_b, reference, models, fmt=case.fmt,
                           alpha=case.alpha)


def _evaluate_all(case: SweepCase, configs: Sequence[SweepConfig], reference: torch.Tensor,
                  evaluate_fn: Optional[Callable[[SweepCase, SweepConfig, torch.Tensor], int]]) -> list[int]:
    if evaluate_fn is not None:
        return [evaluate_fn(case, c, reference) for c in configs]
    out = [0] * len(configs)
    batch = [i for i, c in enumerate(configs) if c.w_reduce in BATCH_W_REDUCE]
    if batch:
        for i, n in zip(batch, evaluate_batch(case, [configs[i] for i in batch], reference)):
            out[i] = n
    for i, c in enumerate(configs):
        if c.w_reduce not in BATCH_W_REDUCE:
            out[i] = evaluate(case, c, reference)
    return out


def run_sweep(case: SweepCase, reference: torch.Tensor, configs: Sequence[SweepConfig],
              evaluate_fn: Optional[Callable[[SweepCase, SweepConfig, torch.Tensor], int]] = None) -> list[int]:
    """Mismatch count per configuration, on this process's device (evaluate_fn: a per-model evaluator
    to use instead of the batched kernel)."""
    return _evaluate_all(case, configs, reference, evaluate_fn)


def _broadcast(t: torch.Tensor, src: int, group, comm_dev) -> torch.Tensor:
    import torch.distributed as dist

    x = t.to(comm_dev).contiguous()
    dist.broadcast(x, src=src, group=group)
    return x


def run_sweep_sharded(case: Optional[SweepCase], reference: Optional[torch.Tensor], configs: Sequence[SweepConfig],
                      *, group=None,
                      evaluate_fn: Optional[Callable[[SweepCase, SweepConfig, torch.Tensor], int]] = None) -> list[int]:
    """run_sweep over all ranks of the default (or given) process group; same call on every rank.
    Rank 0 passes the case and the reference (the other ranks' arguments are ignored): their shapes
    travel first (broadcast_object_list), then the tensors.  Returns the full mismatch list on every
    rank."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    comm_dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    meta = [None]
    if rank == 0:
        tensors = [case.a_fp4, case.b_fp4, case.scale_a, case.scale_b, reference]
        if case.alpha is not None:
            tensors.append(case.alpha)
        meta = [(case.fmt, [(tuple(t.shape), t.dtype) for t in tensors])]
    dist.broadcast_object_list(meta, src=0, group=group)
    fmt, shapes = meta[0]
    if rank != 0:
        tensors = [torch.empty(sh, dtype=dt, device=comm_dev) for sh, dt in shapes]
    tensors = [_broadcast(t, 0, group, comm_dev) for t in tensors]
    local = SweepCase(tensors[0], tensors[1], tensors[2], tensors[3], fmt, tensors[5] if len(tensors) > 5 else None)
    reference = tensors[4]
    table = torch.zeros((len(configs), 2), dtype=torch.int64)
    mine = list(range(rank, len(configs), world))
    for i, n in zip(mine, _evaluate_all(local, [configs[i] for i in mine], reference, evaluate_fn)):
        table[i, 0] = n
        table[i, 1] = 1
    t = table.to(comm_dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    t = t.cpu()
    if int(t[:, 1].sum()) != len(configs):
        raise RuntimeError("sweep: not every configuration was evaluated")
    return [int(x) for x in t[:, 0]]
