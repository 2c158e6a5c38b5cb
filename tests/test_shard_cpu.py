"""Host logic of the one-GEMM split over ranks (no GPU): the column and tile partitions, the row slices
in the swizzled scale layout, and the gather of the output over two gloo ranks (columns) and four (a
2 x 2 grid of tiles), with the C oracle computing each rank's share -- the gathered output must equal
the oracle's whole GEMM bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from emugen_b200 import shard


@pytest.mark.parametrize("n,world", [(8192, 1), (8192, 2), (8192, 8), (300, 2), (1000, 3), (128, 4), (5, 2)])
def test_column_ranges_cover_in_order_and_align(n, world):
    ranges = [shard.column_range(n, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for a0, a1 in ranges:
        assert a0 <= a1 and (a0 % 128 == 0 or a0 == n)
    units = [-(-(a1 - a0) // 128) for a0, a1 in ranges]   # 128-row blocks per rank: balanced to within one
    assert max(units) - min(units) <= 1


def _problem():
    from tests.golden.make_golden import gen_inputs

    case = dict(kind="nvfp", data="normal", M=40, N=300, K=256, r3=0, r4=0, out=0)
    a, b, sfa, sfb, alpha = gen_inputs(case, np.random.default_rng(3))
    return a, b, sfa, sfb, float(alpha)


def _oracle(a, b, sfa, sfb, alpha):
    from oracle import oracle

    return oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0, group_size=16, w_reduce=4, alpha=alpha)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, b, sfa, sfb, alpha = _problem()
        n0, n1 = shard.column_range(b.shape[0], world, rank)
        bq, bs = shard.b_slice(torch.from_numpy(b), torch.from_numpy(sfb), n0, n1)
        local = _oracle(a, bq.numpy(), sfa, bs.numpy(), alpha)
        full = shard.gather_columns(torch.from_numpy(local.view(np.float16)), b.shape[0])   # bits carried as fp16
        results[rank] = bool(np.array_equal(full.numpy().view(np.uint16), _oracle(a, b, sfa, sfb, alpha)))
    finally:
        dist.destroy_process_group()


def test_split_gemm_gathers_to_the_whole_gemm_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        assert all(p.exitcode == 0 for p in procs)
        assert dict(results) == {0: True, 1: True}


@pytest.mark.parametrize("world", [1, 2, 3, 4, 6, 8])
def test_tile_grid_covers_the_output_once(world):
    pr, pc = shard.grid_shape(world)
    assert pr * pc == world and (pr == 1 or world >= 4)
    m, n = 8192 + 300, 8192 + 40
    cover = np.zeros((m // 64 + 8, n // 64 + 8), dtype=np.int32)
    for r in range(world):
        (m0, m1), (n0, n1) = shard.tile_ranges(m, n, world, r)
        assert m0 % 128 == 0 and n0 % 128 == 0
        cover[m0 // 64:-(-m1 // 64), n0 // 64:-(-n1 // 64)] += 1
    assert np.all(cover[: -(-m // 64), : -(-n // 64)] == 1)


def _tile_problem():
    from tests.golden.make_golden import gen_inputs

    case = dict(kind="nvfp", data="normal", M=300, N=600, K=256, r3=0, r4=0, out=0)
    a, b, sfa, sfb, alpha = gen_inputs(case, np.random.default_rng(4))
    return a, b, sfa, sfb, float(alpha)


def _tile_rank_main(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, b, sfa, sfb, alpha = _tile_problem()
        M, N = a.shape[0], b.shape[0]
        (m0, m1), (n0, n1) = shard.tile_ranges(M, N, world, rank)
        aq, as_ = shard.row_slice(torch.from_numpy(a), torch.from_numpy(sfa), m0, m1)
        bq, bs = shard.row_slice(torch.from_numpy(b), torch.from_numpy(sfb), n0, n1)
        local = _oracle(aq.numpy(), bq.numpy(), as_.numpy(), bs.numpy(), alpha)
        full = shard.gather_tiles(torch.from_numpy(local.view(np.float16)), M, N)   # bits carried as fp16
        results[rank] = bool(np.array_equal(full.numpy().view(np.uint16), _oracle(a, b, sfa, sfb, alpha)))
    finally:
        dist.destroy_process_group()


def test_tile_split_gathers_to_the_whole_gemm_on_four_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_tile_rank_main, args=(r, 4, port, results)) for r in range(4)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
        assert all(p.exitcode == 0 for p in procs)
        assert dict(results) == {r: True for r in range(4)}
