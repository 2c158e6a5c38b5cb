"""Randomised real-vs-emulated GEMM suite with the comparison on the device, on one GPU or sharded.

``run_suite`` mirrors gemm_compare/runner.py:171-296 (same arguments, printout and return code)
with ``run_test_case`` (runner.py:82-124) comparing through ``emugen_b200.compare`` (counted on the
device).  ``run_suite_sharded`` runs the same cases over the ranks of an initialised
``torch.distributed`` group: the case list (shapes and distributions) is drawn up front from the
seed on every rank, case i runs on rank i % world with its tensors drawn from a generator seeded by
(seed, i), and the per-case results meet in one ``all_reduce(SUM)``.

``DataGenerator`` / ``DataGenerator_Abs`` restate gemm_compare/data.py:5-56 (same distribution
names and formulas), plus "student_t" (Student-t, 3 degrees of freedom) for the MXFP4 suite.
"""
from __future__ import annotations

import random
import sys
import time
import traceback
from typing import Any, Callable

import torch

from .compare import compare_mse, compare_tensors

QuantFn = Callable[[torch.Tensor, torch.Tensor], Any]
GemmFn = Callable[[Any], torch.Tensor]


def _randn(shape, device, dtype, generator):
    return torch.randn(shape, generator=generator, dtype=torch.float32).to(device=device, dtype=dtype) \
        if generator is not None else torch.randn(shape, device=device, dtype=dtype)


def _rand(shape, device, dtype, generator):
    return torch.rand(shape, generator=generator, dtype=torch.float32).to(device=device, dtype=dtype) \
        if generator is not None else torch.rand(shape, device=device, dtype=dtype)


class DataGenerator:
    """Signed test distributions.  ``generator`` (a CPU torch.Generator) makes a draw reproducible
    across devices; without it the device's default generator is used, as the reference does."""

    @staticmethod
    def get_random_tensor(shape, dist_type, device="cuda", dtype=torch.float16, generator=None):
        if dist_type == "normal":
            return _randn(shape, device, dtype, generator)
        if dist_type == "uniform":
            return _rand(shape, device, dtype, generator) * 2 - 1
        if dist_type == "large":
            return _randn(shape, device, dtype, generator) * 100.0
        if dist_type == "small":
            return _randn(shape, device, dtype, generator) * 0.001
        if dist_type == "outliers":
            t = _randn(shape, device, dtype, generator)
            mask = _rand(shape, device, torch.float32, generator) < 0.01
            t[mask] *= 50.0
            return t
        if dist_type == "mixed_rows":
            t = _randn(shape, device, dtype, generator)
            scale = torch.exp(_randn((shape[0], 1), device, torch.float32, generator) * 2)
            return t * scale.to(dtype)
        if dist_type == "abs_large":
            return torch.abs(_randn(shape, device, dtype, generator)) * 100.0
        if dist_type == "student_t":
            d = torch.distributions.StudentT(torch.tensor(3.0))
            if generator is not None:
                # StudentT has no generator argument: draw it as normal / sqrt(chi2 / df) by hand
                z = torch.randn(shape, generator=generator)
                c = torch.zeros(shape)
                for _ in range(3):
                    c += torch.randn(shape, generator=generator) ** 2
                return (z / torch.sqrt(c / 3.0)).to(device=device, dtype=dtype)
            return d.sample(shape).to(device=device, dtype=dtype)
        raise ValueError(f"Unknown distribution type: {dist_type}")


class DataGenerator_Abs:
    """Positive-only variants."""

    @staticmethod
    def get_random_tensor(shape, dist_type, device="cuda", dtype=torch.float16, generator=None):
        if dist_type in ("uniform",):
            return _rand(shape, device, dtype, generator)
        if dist_type == "mixed_rows":
            t = torch.abs(_randn(shape, device, dtype, generator))
            scale = torch.exp(_randn((shape[0], 1), device, torch.float32, generator) * 2)
            return t * scale.to(dtype)
        if dist_type == "outliers":
            t = torch.abs(_randn(shape, device, dtype, generator))
            mask = _rand(shape, device, torch.float32, generator) < 0.01
            t[mask] *= 50.0
            return t
        return torch.abs(DataGenerator.get_random_tensor(shape, dist_type, device, dtype, generator))


def run_test_case(iter_idx: int, M: int, N: int, K: int, dist_a: str, dist_b: str, quant_fn: QuantFn,
                  real_fn: GemmFn, emul_fn: GemmFn, *, sample_count: int = 5, device: str = "cuda",
                  dtype: torch.dtype = torch.float16, data_gen=DataGenerator, extra_meta: dict | None = None,
                  metric_mode: str = "exact", generator=None, compare_fn=compare_tensors,
                  mse_fn=compare_mse) -> dict[str, Any]:
    a = data_gen.get_random_tensor((M, K), dist_a, device=device, dtype=dtype, generator=generator)
    b = data_gen.get_random_tensor((N, K), dist_b, device=device, dtype=dtype, generator=generator)
    state = quant_fn(a, b)
    real_output = real_fn(state)
    modeling_res = emul_fn(state)
    if metric_mode == "exact":
        cmp = compare_fn(real_output, modeling_res, sample_count=sample_count)
    elif metric_mode == "mse":
        cmp = mse_fn(real_output, modeling_res)
    else:
        raise ValueError(f"unknown metric_mode={metric_mode!r}")
    out: dict[str, Any] = {"iter": iter_idx, "M": M, "N": N, "K": K, "dist_a": dist_a, "dist_b": dist_b, **cmp}
    if extra_meta:
        out["extra"] = extra_meta
    return out


DEFAULT_DISTRIBUTIONS = ["normal", "uniform", "large", "outliers", "mixed_rows", "abs_large"]


def _draw_cases(seed: int, n: int, distributions, dims_m, dims_n, dims_k):
    rng = random.Random(seed)
    return [(rng.choice(dims_m), rng.choice(dims_n), rng.choice(dims_k), rng.choice(distributions),
             rng.choice(distributions)) for _ in range(n)]


def _summary(name: str, total: int, results: list[dict[str, Any]], metric_mode: str) -> int:
    print("\n" + "=" * 70)
    print(f"SUMMARY | {name}")
    print("=" * 70)
    if metric_mode == "mse":
        total_numel = sum(int(r.get("mse_numel", 0)) for r in results)
        total_mse_sum = sum(float(r.get("mse_sum", 0.0)) for r in results)
        per_gemm = [float(r.get("per_gemm_rel_l2_error", 0.0)) for r in results]
        print(f"Total: {total}, Completed: {len(results)}")
        print(f"MSE mean: {total_mse_sum / max(total_numel, 1):.8e}")
        print(f"mean over GEMMs of sqrt(sum(error^2)) / sqrt(sum(real^2)): {sum(per_gemm) / max(len(per_gemm), 1):.8e}")
        print(f"MSE max (worst element): {max((float(r.get('max_mse', 0.0)) for r in results), default=0.0):.8e}")
        return 0
    mismatches = [r for r in results if r["status"] == "MISMATCH"]
    print(f"Total: {total}, Matches: {len(results) - len(mismatches)}, Mismatches: {len(mismatches)}")
    print("=" * 70)
    if not mismatches:
        print("*** All tests: exact bitwise match ***")
        return 0
    print(f"Exact-match rate: {(len(results) - len(mismatches)) / max(len(results), 1) * 100:.2f}%")
    return 1


def run_suite(quant_fn: QuantFn, real_fn: GemmFn, emul_fn: GemmFn, *, name: str = "GEMM compare",
              num_iterations: int = 100, distributions: list[str] | None = None, dims_m: list[int] | None = None,
              dims_n: list[int] | None = None, dims_k: list[int] | None = None, sample_count: int = 5,
              max_mismatch_print: int = 20, device: str = "cuda", dtype: torch.dtype = torch.float16,
              data_gen=DataGenerator, seed: int | None = None, metric_mode: str = "exact",
              print_iter_status: bool = True, compare_fn=compare_tensors, mse_fn=compare_mse) -> int:
    """Randomised suite; returns 0 when every case matches exactly (or in MSE mode), else 1."""
    if seed is None:
        seed = int(time.time() * 1e6) ^ int.from_bytes(__import__("os").urandom(8), "little")
    random.seed(seed)
    torch.manual_seed(seed)
    if device == "cuda" and torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    print("seed =", seed)
    distributions = distributions or DEFAULT_DISTRIBUTIONS
    dims_m = dims_m or [128, 256, 1024, 2048, 4096]
    dims_n = dims_n or [128, 256, 1024, 2048, 4096]
    dims_k = dims_k or [128, 256, 512, 1024]
    print(f"\n{'=' * 70}\n{name}\n{'=' * 70}")
    print(f"Iterations: {num_iterations}")
    print(f"Distributions: {distributions}")
    print(f"Dims M: {dims_m} | N: {dims_n} | K: {dims_k}")
    print("=" * 70)
    results: list[dict[str, Any]] = []
    printed = 0
    for i in range(num_iterations):
        M, N, K = random.choice(dims_m), random.choice(dims_n), random.choice(dims_k)
        da, db = random.choice(distributions), random.choice(distributions)
        print(f"\rTest {i + 1}/{num_iterations}: K={K:4}, A={da:10}, B={db:10} ... ", end="")
        sys.stdout.flush()
        try:
            res = run_test_case(i, M, N, K, da, db, quant_fn, real_fn, emul_fn, sample_count=sample_count,
                                device=device, dtype=dtype, data_gen=data_gen, metric_mode=metric_mode,
                                compare_fn=compare_fn, mse_fn=mse_fn)
            results.append(res)
            print(res["status"] if print_iter_status else "OK")
            if metric_mode == "exact" and res["status"] == "MISMATCH" and printed < max_mismatch_print:
                printed += 1
                print("    >>> Mismatch Details:")
                for d in res["mismatch_details"]:
                    print(f"      Pos {d['idx']}: Real={d['real']:.6f} | Model={d['model']:.6f} | Diff={d['diff']:.6f}")
        except Exception as e:  # reported per case, as the reference does
            print(f"\nFATAL ERROR on Test {i + 1}: {e}")
            traceback.print_exc()
    return _summary(name, num_iterations, results, metric_mode)


def run_suite_sharded(quant_fn: QuantFn, real_fn: GemmFn, emul_fn: GemmFn, *, seed: int,
                      name: str = "GEMM compare (sharded)", num_iterations: int = 100,
                      distributions: list[str] | None = None, dims_m: list[int] | None = None,
                      dims_n: list[int] | None = None, dims_k: list[int] | None = None, device: str = "cuda",
                      dtype: torch.dtype = torch.float16, data_gen=DataGenerator, metric_mode: str = "exact",
                      compare_fn=compare_tensors, mse_fn=compare_mse, group=None) -> int:
    """run_suite over all ranks of the default (or given) process group; same code on every rank."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    cases = _draw_cases(seed, num_iterations, distributions or DEFAULT_DISTRIBUTIONS,
                        dims_m or [128, 256, 1024, 2048, 4096], dims_n or [128, 256, 1024, 2048, 4096],
                        dims_k or [128, 256, 512, 1024])
    table = torch.zeros((num_iterations, 6), dtype=torch.float64)   # done, mismatch, max, sum, numel, ref sq
    for i in range(rank, num_iterations, world):
        M, N, K, da, db = cases[i]
        g = torch.Generator().manual_seed((seed * 1000003 + i) & 0x7FFFFFFFFFFFFFFF)
        try:
            r = run_test_case(i, M, N, K, da, db, quant_fn, real_fn, emul_fn, device=device, dtype=dtype,
                              data_gen=data_gen, metric_mode=metric_mode, generator=g, compare_fn=compare_fn,
                              mse_fn=mse_fn)
        except Exception as e:
            print(f"[rank {rank}] FATAL ERROR on Test {i + 1}: {e}", file=sys.stderr)
            continue
        table[i, 0] = 1.0
        if metric_mode == "exact":
            table[i, 1] = 1.0 if r["status"] == "MISMATCH" else 0.0
            table[i, 2] = float(r["max_diff"])
        else:
            table[i, 3], table[i, 4], table[i, 5] = float(r["mse_sum"]), float(r["mse_numel"]), float(r["real_sq_sum"])
            table[i, 2] = float(r["max_mse"])
    comm_dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    t = table.to(comm_dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    table = t.cpu()
    results: list[dict[str, Any]] = []
    for i in range(num_iterations):
        if table[i, 0] == 0:
            continue
        if metric_mode == "exact":
            results.append({"status": "MISMATCH" if table[i, 1] > 0 else "SUCCESS", "max_diff": float(table[i, 2])})
        else:
            s, ne, rs = float(table[i, 3]), int(table[i, 4]), float(table[i, 5])
            results.append({"status": "OK", "mse_sum": s, "mse_numel": ne, "real_sq_sum": rs,
                            "max_mse": float(table[i, 2]), "per_gemm_rel_l2_error": s ** 0.5 / max(rs ** 0.5, 1e-12)})
    if rank == 0:
        return _summary(name, num_iterations, results, metric_mode)
    if metric_mode == "mse":
        return 0
    return 1 if any(r["status"] == "MISMATCH" for r in results) else 0
