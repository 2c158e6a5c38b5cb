"""One emulated GEMM split over the ranks of a process group by output columns.

The reference computes one ``emulated_scaled_fp4_mm`` call as a loop over M chunks
(nvfp_emulation.cpp:115); its output columns are as independent as its rows.  Here rank r of W owns a
contiguous range of output columns -- rows [n0, n1) of B -- and computes C[:, n0:n1] from all of A:
no exchange in the GEMM itself.  Column ranges are whole 128-row blocks of B, because the 128x4
swizzled scale layout keeps each block of 128 rows contiguous, so a rank's B operand is a plain slice
of the packed values and of the scale buffer.

The one exchange of the NVFP4 path comes before the GEMM: the global scale of an operand is taken
from its amax over ALL of it (gemm_compare/backends/nvfp.py:24-27), so ranks holding shards combine
their amax words with one all_reduce(MAX) of two int32 words (``sharded_global_scales``).
``gather_columns`` assembles C on every rank with one all_gather when the caller wants it whole.
"""
from __future__ import annotations

import torch

from . import _lib

ROW_BLOCK = 128   # rows of one swizzled scale block


def column_range(n: int, world: int, rank: int, align: int = ROW_BLOCK) -> tuple[int, int]:
    """Rank `rank`'s output columns [n0, n1) of an N-column GEMM: contiguous, n0 a multiple of
    `align`, the ranges of ranks 0..world-1 in order covering [0, n) (later ranks may be empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    units = -(-n // align)
    per, extra = divmod(units, world)
    u0 = rank * per + min(rank, extra)
    u1 = u0 + per + (1 if rank < extra else 0)
    return min(n, u0 * align), min(n, u1 * align)


def b_slice(b_fp4: torch.Tensor, scale_b: torch.Tensor, n0: int, n1: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows [n0, n1) of B: its packed values and the scale rows of the 128-row blocks they occupy
    (n0 a multiple of 128; the slice stays in the swizzled layout, zero-padded rows included)."""
    if n0 % ROW_BLOCK:
        raise ValueError(f"n0 = {n0} is not a multiple of {ROW_BLOCK}")
    rows = -(-(n1 - n0) // ROW_BLOCK) * ROW_BLOCK
    return b_fp4[n0:n1], scale_b[n0:n0 + rows]


def sharded_global_scales(a: torch.Tensor, b: torch.Tensor, *, a_sharded: bool, b_sharded: bool, group=None):
    """NVFP4 (gs_a, gs_b, alpha) of operands of which this rank holds `a` and `b` -- the whole operand
    or its shard, as flagged -- equal to emu_nvfp4_global_scales on the whole operands.  One
    all_reduce(MAX) of the two amax words when either operand is sharded."""
    import torch.distributed as dist

    words = _lib.nvfp4_amax(a, b)
    if a_sharded or b_sharded:
        mine = words.clone()
        dist.all_reduce(words, op=dist.ReduceOp.MAX, group=group)
        if not a_sharded:
            words[0:1].copy_(mine[0:1])
        if not b_sharded:
            words[1:2].copy_(mine[1:2])
    return _lib.nvfp4_scales_from_amax(words)


def gather_columns(c_local: torch.Tensor, n: int, group=None) -> torch.Tensor:
    """All ranks' column slices (from column_range) assembled into the full [M, n] output on every
    rank, with one all_gather of equally padded slices."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    widths = [b - a for a, b in (column_range(n, world, r) for r in range(world))]
    w = max(widths)
    m = c_local.shape[0]
    padded = torch.zeros((m, w), dtype=c_local.dtype, device=c_local.device)
    padded[:, :c_local.shape[1]] = c_local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    return torch.cat([p[:, :wd] for p, wd in zip(parts, widths)], dim=1)
