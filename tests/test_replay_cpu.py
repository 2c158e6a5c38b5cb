"""Host logic of rollout replay (no GPU): the artefact format round trip, the single-process replay
return codes, and the sharded replay over two gloo ranks (per-case results reduced with one
all_reduce, same return code on every rank)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from emugen_b200 import replay
from emugen_b200.backends.nvfp import NVFPQuantState, nvfp_quant_state_to_cpu_dict

BAD_ALPHA = 0.125   # the case whose emulation is perturbed by the fake emulator below


def _fake_gemm(state):
    """Deterministic CPU stand-in for the emulated GEMM (the replay logic under test is GPU-free)."""
    out = (state.a_fp4.float() @ state.b_fp4.float().T / 64.0).to(state.out_dtype)
    if abs(float(state.alpha.reshape(-1)[0]) - BAD_ALPHA) < 1e-9:
        out = out.clone()
        out[1, 2] = out[1, 2] * 2 + 1
    return out


def _cpu_compare(real, model, *, sample_count=5):
    diff = (real.float() - model.float()).abs()
    diff[real == model] = 0.0
    diff[real.isnan() & model.isnan()] = 0.0
    diff[diff.isnan()] = float("inf")
    m = diff.max().item()
    return {"status": "SUCCESS" if m == 0 else "MISMATCH", "max_diff": m, "mismatch_details": []}


def _cpu_mse(ref, tgt):
    sq = torch.nan_to_num((ref.float() - tgt.float()).pow(2), nan=0.0, posinf=0.0, neginf=0.0)
    rs = torch.nan_to_num(ref.float().pow(2), nan=0.0, posinf=0.0, neginf=0.0).sum().item()
    s = sq.sum().item()
    return {"status": "OK", "mean_mse": s / sq.numel(), "max_mse": sq.max().item(), "mse_sum": s,
            "mse_numel": sq.numel(), "real_sq_sum": rs, "per_gemm_rel_l2_error": s ** 0.5 / max(rs ** 0.5, 1e-12),
            "mismatch_details": []}


def _make_artifact(path, n_cases=5, bad=(3,)):
    g = torch.Generator().manual_seed(0)
    cases = []
    for i in range(n_cases):
        M, N, K = 8 + i, 16, 64
        st = NVFPQuantState(
            a_fp4=torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.uint8),
            b_fp4=torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8),
            scale_a=torch.zeros(128, 4, dtype=torch.uint8).view(torch.float8_e4m3fn),
            scale_b=torch.zeros(128, 4, dtype=torch.uint8).view(torch.float8_e4m3fn),
            global_scale_a=torch.ones(1), global_scale_b=torch.ones(1),
            alpha=torch.tensor([BAD_ALPHA if i in bad else 1.0 + i]), out_dtype=torch.float16,
            w_reduce=4, group_size=16, m_chunk_size=128, stage3_rounding=0, stage4_rounding=0)
        real = (st.a_fp4.float() @ st.b_fp4.float().T / 64.0).to(torch.float16)
        cases.append({"iter": i, "M": M, "N": N, "K": K, "dist_a": "normal", "dist_b": "normal",
                      "state": nvfp_quant_state_to_cpu_dict(st), "real_output": real})
    write_rollout(path, backend="nvfp", meta={"note": "test"}, seed=7, cases=cases)


def write_rollout(path, *, backend, cases, seed=0, meta=None, version=1):
    """An artefact in the format the reference's export harness writes (gemm_compare/rollout.py:48-79)."""
    torch.save({"gemm_compare_rollout_version": version, "backend": backend, "meta": meta or {}, "seed": seed,
                "cases": cases}, path)


def test_artifact_reader(tmp_path):
    p = tmp_path / "r.pt"
    _make_artifact(p)
    r = replay.Rollout.read(p)
    assert r.backend == "nvfp" and r.seed == 7 and r.meta == {"note": "test"} and len(r.cases) == 5
    st = r.state(0, device="cpu")
    assert st.a_fp4.shape == (8, 32) and st.out_dtype == torch.float16
    bad = tmp_path / "bad.pt"
    write_rollout(bad, backend="nvfp", cases=[], version=99)
    with pytest.raises(ValueError, match="version 99"):
        replay.Rollout.read(bad)
    write_rollout(bad, backend="nvfp", cases=[{"M": 1}])
    with pytest.raises(ValueError, match="case 0 lacks state"):
        replay.Rollout.read(bad)
    torch.save([1, 2], bad)
    with pytest.raises(ValueError, match="not a rollout"):
        replay.Rollout.read(bad)
    # an unreadable artefact is reported as code 2, like a backend mismatch
    assert replay.run_suite_import(_fake_gemm, backend="nvfp", artifact_path=bad, device="cpu") == 2


def test_single_process_replay_codes(tmp_path):
    p = tmp_path / "r.pt"
    _make_artifact(p, bad=())
    kw = dict(backend="nvfp", artifact_path=p, device="cpu", compare_fn=_cpu_compare, mse_fn=_cpu_mse)
    assert replay.run_suite_import(_fake_gemm, **kw) == 0
    _make_artifact(p, bad=(2,))
    assert replay.run_suite_import(_fake_gemm, **kw) == 1
    assert replay.run_suite_import(_fake_gemm, metric_mode="mse", **kw) == 0
    assert replay.run_suite_import(_fake_gemm, **{**kw, "backend": "mxfp"}) == 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path, metric_mode, backend, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rc = replay.run_suite_import_sharded(_fake_gemm, backend=backend, artifact_path=path, device="cpu",
                                             metric_mode=metric_mode, compare_fn=_cpu_compare, mse_fn=_cpu_mse)
        results[rank] = rc
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("metric_mode,backend,bad,expect", [
    ("exact", "nvfp", (), 0), ("exact", "nvfp", (1, 4), 1), ("mse", "nvfp", (1,), 0), ("exact", "mxfp", (), 2)])
def test_sharded_replay_two_gloo_ranks(tmp_path, metric_mode, backend, bad, expect):
    p = tmp_path / "r.pt"
    _make_artifact(p, n_cases=7, bad=bad)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(p), metric_mode, backend, results))
                 for r in range(2)]
        for pr in procs:
            pr.start()
        for pr in procs:
            pr.join(timeout=120)
        assert all(pr.exitcode == 0 for pr in procs)
        assert dict(results) == {0: expect, 1: expect}
