"""Host logic of the randomised suite (no GPU): the distributions, the single-process suite and the
sharded suite over two gloo ranks agree on the verdict (fake GEMMs on CPU, CPU comparison)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from emugen_b200 import suite


def _quant(a, b):
    return (a, b)


def _real(st):
    a, b = st
    return (a.float() @ b.float().T).half()


def _emul_bad(st):
    out = _real(st)
    a, _ = st
    if a.shape[1] == 256:           # every K = 256 case mismatches
        out = out.clone()
        out[0, 0] = out[0, 0] * 2 + 1
    return out


def _cmp(real, model, *, sample_count=5):
    bad = ~((real == model) | (real.isnan() & model.isnan()))
    diff = (real.float() - model.float()).abs()
    m = float(diff[bad].max()) if bad.any() else 0.0
    return {"status": "MISMATCH" if bad.any() else "SUCCESS", "max_diff": m, "mismatch_details": []}


def _mse(ref, tgt):
    sq = torch.nan_to_num((ref.float() - tgt.float()).pow(2), nan=0.0, posinf=0.0, neginf=0.0)
    rs = float(torch.nan_to_num(ref.float().pow(2), nan=0.0, posinf=0.0, neginf=0.0).sum())
    return {"status": "OK", "mean_mse": float(sq.mean()), "max_mse": float(sq.max()), "mse_sum": float(sq.sum()),
            "mse_numel": sq.numel(), "real_sq_sum": rs, "per_gemm_rel_l2_error": float(sq.sum()) ** 0.5 / max(rs ** 0.5, 1e-12),
            "mismatch_details": []}


KW = dict(num_iterations=9, dims_m=[8, 16], dims_n=[8, 24], dims_k=[128, 256], device="cpu", dtype=torch.float32,
          compare_fn=_cmp, mse_fn=_mse)


@pytest.mark.parametrize("dist_name", ["normal", "uniform", "large", "small", "outliers", "mixed_rows", "abs_large",
                                       "student_t"])
def test_distributions_shape_and_reproducibility(dist_name):
    for gen in (suite.DataGenerator, suite.DataGenerator_Abs):
        g1, g2 = torch.Generator().manual_seed(3), torch.Generator().manual_seed(3)
        x = gen.get_random_tensor((16, 32), dist_name, device="cpu", dtype=torch.float32, generator=g1)
        y = gen.get_random_tensor((16, 32), dist_name, device="cpu", dtype=torch.float32, generator=g2)
        assert x.shape == (16, 32) and torch.equal(x, y)
        if gen is suite.DataGenerator_Abs:
            assert (x >= 0).all()


def test_single_process_suite_codes():
    assert suite.run_suite(_quant, _real, _real, seed=11, **KW) == 0
    cases = suite._draw_cases(11, 9, suite.DEFAULT_DISTRIBUTIONS, [8, 16], [8, 24], [128, 256])
    expect_bad = any(c[2] == 256 for c in cases)
    assert suite.run_suite(_quant, _real, _emul_bad, seed=11, **KW) == (1 if expect_bad else 0)
    assert suite.run_suite(_quant, _real, _emul_bad, seed=11, metric_mode="mse", **KW) == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, bad, mode, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        results[rank] = suite.run_suite_sharded(_quant, _real, _emul_bad if bad else _real, seed=11,
                                                metric_mode=mode, **KW)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bad,mode", [(False, "exact"), (True, "exact"), (True, "mse")])
def test_sharded_suite_two_gloo_ranks(bad, mode):
    cases = suite._draw_cases(11, 9, suite.DEFAULT_DISTRIBUTIONS, [8, 16], [8, 24], [128, 256])
    expect = 1 if (bad and mode == "exact" and any(c[2] == 256 for c in cases)) else 0
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, bad, mode, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        assert all(p.exitcode == 0 for p in procs)
        assert dict(results) == {0: expect, 1: expect}
