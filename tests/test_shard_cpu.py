"""Host logic of the one-GEMM split over ranks (no GPU): the column partition, the B slice in the
swizzled scale layout, and the gather of the output over two gloo ranks, with the C oracle computing
each rank's columns -- the gathered output must equal the oracle's whole GEMM bit for bit."""
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
