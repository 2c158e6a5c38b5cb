"""One emulated GEMM split over the ranks of a process group by output tiles.

The reference computes one ``emulated_scaled_fp4_mm`` call as a loop over M chunks
(nvfp_emulation.cpp:115); its outputs are independent of each other.  Here the W ranks form a grid of
pr x pc (``grid_shape``: 1 x 2 for two ranks, 2 x W/2 for four and eight) and rank r = ri * pc + ci owns
rows [m0, m1) of A and rows [n0, n1) of B and computes C[m0:m1, n0:n1]: no exchange in the GEMM
itself.  Every per-operand cost that does not shrink with the columns (A's quantisation and the GEMM's
per-row pre-pass) is then split over pr ranks instead of repeated on all of them.  Row ranges are whole
128-row blocks, because the 128x4 swizzled scale layout keeps each block of 128 rows contiguous, so a
rank's operands are plain slices of the packed values and of the scale buffers.

The one exchange of the NVFP4 path comes before the GEMM: the global scale of an operand is taken
from its amax over ALL of it (gemm_compare/backends/nvfp.py:24-27), so ranks holding shards combine
their amax words with one all_reduce(MAX) of two int32 words (``sharded_global_scales``).
``gather_tiles`` (``gather_columns`` for a one-row grid) assembles C on every rank with one all_gather when
the caller wants it whole.
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


def grid_shape(world: int) -> tuple[int, int]:
    """(row shards pr, column shards pc) of a W-rank split: columns only for up to three ranks (A's
    per-row work is about the size of B's per-row work, and a one-row grid needs no A exchange at all),
    2 x W/2 for an even W of four or more."""
    if world < 1:
        raise ValueError(f"world {world}")
    return (2, world // 2) if world >= 4 and world % 2 == 0 else (1, world)


def tile_ranges(m: int, n: int, world: int, rank: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """Rank `rank`'s output tile: rows [m0, m1) of A and rows [n0, n1) of B (column_range on each axis of
    grid_shape(world); rank = row index * pc + column index)."""
    pr, pc = grid_shape(world)
    ri, ci = divmod(rank, pc)
    return column_range(m, pr, ri), column_range(n, pc, ci)


def row_slice(x_fp4: torch.Tensor, scale: torch.Tensor, r0: int, r1: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows [r0, r1) of a packed operand (A or B): its packed values and the scale rows of the 128-row
    blocks they occupy (r0 a multiple of 128; the slice stays in the swizzled layout, zero-padded rows
    included)."""
    if r0 % ROW_BLOCK:
        raise ValueError(f"row {r0} is not a multiple of {ROW_BLOCK}")
    rows = -(-(r1 - r0) // ROW_BLOCK) * ROW_BLOCK
    return x_fp4[r0:r1], scale[r0:r0 + rows]


def b_slice(b_fp4: torch.Tensor, scale_b: torch.Tensor, n0: int, n1: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows [n0, n1) of B (row_slice)."""
    return row_slice(b_fp4, scale_b, n0, n1)


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


def gather_tiles(c_local: torch.Tensor, m: int, n: int, group=None) -> torch.Tensor:
    """All ranks' output tiles (from tile_ranges) assembled into the full [m, n] output on every rank,
    with one all_gather of equally padded tiles."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    ranges = [tile_ranges(m, n, world, r) for r in range(world)]
    h = max(m1 - m0 for (m0, m1), _ in ranges)
    w = max(n1 - n0 for _, (n0, n1) in ranges)
    padded = torch.zeros((h, w), dtype=c_local.dtype, device=c_local.device)
    padded[:c_local.shape[0], :c_local.shape[1]] = c_local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    full = torch.empty((m, n), dtype=c_local.dtype, device=c_local.device)
    for p, ((m0, m1), (n0, n1)) in zip(parts, ranges):
        full[m0:m1, n0:n1] = p[:m1 - m0, :n1 - n0]
    return full


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
