"""GPU: on-device comparison (emu_compare) against the reference's torch formulation of
compare_tensors / compare_mse, the FP4 dequantiser against flashinfer (MXFP4) and the stated
formula (NVFP4), pseudo_fn, and rollout replay through the emulated GEMM."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_compare(real, model, sample_count=5):
    """gemm_compare/runner.py:20-55 restated with torch ops (the comparison the tests check against)."""
    diff = (real.float() - model.float()).abs()
    diff[real == model] = 0.0
    diff[real.isnan() & model.isnan()] = 0.0
    diff[diff.isnan()] = float("inf")
    m = diff.max().item()
    idx = torch.nonzero(diff != 0, as_tuple=False)[:sample_count].tolist()
    return m, [tuple(i) for i in idx], int((diff != 0).sum().item())


def _ref_mse(ref, tgt):
    sq = torch.nan_to_num((ref.float() - tgt.float()).pow(2), nan=0.0, posinf=0.0, neginf=0.0)
    rs = torch.nan_to_num(ref.float().pow(2), nan=0.0, posinf=0.0, neginf=0.0)
    return sq.double().sum().item(), sq.max().item(), rs.double().sum().item()


def _planted(dtype, shape=(300, 517), seed=0):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(shape, generator=g) * 10).to(dtype)
    b = a.clone()
    flat_a, flat_b = a.view(-1), b.view(-1)
    n = flat_a.numel()
    sel = torch.randperm(n, generator=g)[:40]
    flat_b[sel[:10]] = flat_b[sel[:10]] * 2 + 1              # plain mismatches
    flat_a[sel[10:15]] = float("nan")                          # NaN on one side only
    flat_a[sel[15:20]] = float("nan"); flat_b[sel[15:20]] = float("nan")   # NaN on both: match
    flat_a[sel[20:25]] = 0.0; flat_b[sel[20:25]] = -0.0        # +0 == -0: match
    flat_a[sel[25:28]] = float("inf"); flat_b[sel[25:28]] = 1.0
    flat_a[sel[28:30]] = float("inf"); flat_b[sel[28:30]] = float("inf")   # equal infinities
    return a, b


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_compare_tensors_matches_reference_semantics(dtype):
    from emugen_b200.compare import compare_tensors

    a, b = _planted(dtype)
    got = compare_tensors(a.cuda(), b.cuda(), sample_count=5)
    m, idx, cnt = _ref_compare(a, b)
    assert got["max_diff"] == m and got["status"] == "MISMATCH"
    assert [d["idx"] for d in got["mismatch_details"]] == idx
    from emugen_b200 import _lib

    st = _lib.compare_stats(a.cuda(), b.cuda())
    assert st["mismatches"] == cnt
    assert st["first_index"] == idx[0][0] * a.shape[1] + idx[0][1]
    same = compare_tensors(a.cuda(), a.cuda())
    assert same["status"] == "SUCCESS" and same["max_diff"] == 0 and same["mismatch_details"] == []
    assert _lib.compare_stats(a.cuda(), a.cuda())["first_index"] == -1


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_compare_mse_matches_reference_within_rounding(dtype):
    from emugen_b200.compare import compare_mse

    a, b = _planted(dtype, seed=1)
    got = compare_mse(a.cuda(), b.cuda())
    s, mx, rs = _ref_mse(a, b)
    assert got["max_mse"] == mx
    assert math.isclose(got["mse_sum"], s, rel_tol=1e-12)
    assert math.isclose(got["real_sq_sum"], rs, rel_tol=1e-12)
    assert got["mse_numel"] == a.numel()


def test_compare_large_and_empty():
    from emugen_b200 import _lib

    a = torch.randn(8192, 8192, device="cuda").half()
    b = a.clone()
    b[4095, 17] = -b[4095, 17] - 1
    st = _lib.compare_stats(a, b)
    assert st["mismatches"] == 1 and st["first_index"] == 4095 * 8192 + 17
    e = torch.empty(0, device="cuda", dtype=torch.float16)
    st = _lib.compare_stats(e, e)
    assert st["mismatches"] == 0 and st["first_index"] == -1 and st["numel"] == 0


def test_dequant_mxfp4_matches_flashinfer_bits():
    import flashinfer

    from emugen_b200 import _lib
    from tests.golden.make_golden import pad, swizzle

    rng = np.random.default_rng(3)
    M, K = 200, 512
    q = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    sf = rng.integers(0, 256, (M, K // 32), dtype=np.uint8)
    sf[0, 0], sf[1, 1], sf[2, 2] = 0, 255, 254
    sfz = swizzle(sf, pad(M, 128), pad(K // 32, 4))
    got = _lib.dequant_fp4(torch.from_numpy(q).cuda(), torch.from_numpy(sfz).cuda(), fmt=_lib.EMU_FMT_MXFP4).cpu()
    ref = flashinfer.mxfp4_dequantize(torch.from_numpy(q), torch.from_numpy(sfz))
    g, r = got.numpy().view(np.uint32), ref.float().numpy().view(np.uint32)
    gn, rn = np.isnan(got.numpy()), np.isnan(ref.float().numpy())
    assert np.array_equal(gn, rn) and np.array_equal(g[~gn], r[~rn])


def test_dequant_nvfp4_formula():
    from emugen_b200 import _lib
    from tests.golden.make_golden import pad, swizzle

    rng = np.random.default_rng(4)
    M, K = 130, 256
    q = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    sf = rng.integers(0, 0x7F, (M, K // 16), dtype=np.uint8)
    gs = np.float32(37.5)
    sfz = swizzle(sf, pad(M, 128), pad(K // 16, 4))
    got = _lib.dequant_fp4(torch.from_numpy(q).cuda(), torch.from_numpy(sfz).cuda(), fmt=_lib.EMU_FMT_NVFP4,
                           global_scale=torch.tensor([float(gs)])).cpu().numpy()
    lut = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)
    codes = np.stack([q & 15, q >> 4], -1).reshape(M, K)
    scale = torch.from_numpy(sf).view(torch.float8_e4m3fn).float().numpy() / gs
    ref = (lut[codes] * np.repeat(scale, 16, axis=1)).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("backend", ["nvfp", "mxfp"])
def test_pseudo_fn_is_dequant_then_matmul(backend):
    from emugen_b200.backends.mxfp import build_mxfp_fns
    from emugen_b200.backends.nvfp import build_nvfp_fns

    build = build_nvfp_fns if backend == "nvfp" else build_mxfp_fns
    quant_fn, _real, _emul, pseudo_fn, _meta = build(return_pseudo=True)
    g = torch.Generator().manual_seed(5)
    a = torch.randn(256, 512, generator=g).half().cuda()
    b = torch.randn(128, 512, generator=g).half().cuda()
    st = quant_fn(a, b)
    out = pseudo_fn(st)
    assert out.is_cuda and out.shape == (256, 128)
    ref = (a.float() @ b.float().T)
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    assert rel < 0.2   # FP4 quantisation error, not an exactness check


def test_replay_through_emulated_gemm(tmp_path):
    from emugen_b200 import replay
    from tests.test_replay_cpu import write_rollout
    from emugen_b200.backends.nvfp import build_nvfp_fns, nvfp_quant_state_to_cpu_dict

    quant_fn, _real, emul_fn, _meta = build_nvfp_fns()
    cases = []
    g = torch.Generator().manual_seed(9)
    for i, (M, N, K) in enumerate([(128, 64, 256), (200, 96, 512), (7, 33, 64)]):
        a = torch.randn(M, K, generator=g).half().cuda()
        b = torch.randn(N, K, generator=g).half().cuda()
        st = quant_fn(a, b)
        real = emul_fn(st).cpu()
        if i == 1:
            real[3, 5] = real[3, 5] * 2 + 1
        cases.append({"iter": i, "M": M, "N": N, "K": K, "dist_a": "normal", "dist_b": "normal",
                      "state": nvfp_quant_state_to_cpu_dict(st), "real_output": real})
    p = tmp_path / "roll.pt"
    write_rollout(p, backend="nvfp", cases=cases)
    assert replay.run_suite_import(emul_fn, backend="nvfp", artifact_path=p) == 1
    assert replay.run_suite_import(emul_fn, backend="nvfp", artifact_path=p, metric_mode="mse") == 0
    del cases[1]
    write_rollout(p, backend="nvfp", cases=cases)
    assert replay.run_suite_import(emul_fn, backend="nvfp", artifact_path=p) == 0


@pytest.mark.parametrize("kind,out_mode", [("nvfp", 0), ("mxfp", 1), ("nvfp", 2)])
def test_fused_gemm_compare_matches_separate_compare(kind, out_mode):
    """emu_gemm_compare (comparison in the tensor-core epilogue) against emu_gemm_ws + emu_compare."""
    from emugen_b200 import _lib
    from tests.golden.make_golden import gen_inputs

    case = dict(kind=kind, data="outliers", M=256, N=192, K=1024)
    a, b, sfa, sfb, alpha = gen_inputs(case, np.random.default_rng(21))
    t = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (a, b, sfa, sfb)]
    kw = dict(fmt=0 if kind == "nvfp" else 1, group_size=16 if kind == "nvfp" else 32,
              w_reduce=4 if kind == "nvfp" else 2, stage3_rounding=0, stage4_rounding=0,
              alpha=torch.tensor([float(alpha)], device="cuda") if kind == "nvfp" else None, out_mode=out_mode)
    out = _lib.gemm(*t, **kw)
    ref = out.clone()
    flat = ref.view(-1)
    flat[7] = flat[7] * 2 + 1
    flat[1000] = float("nan")
    flat[5000] = -flat[5000] if flat[5000] != 0 else 1.0
    for path in ("tc", "simt"):
        for write_out in (False, True):
            st, o = _lib.gemm_compare(*t, ref, path=path, write_out=write_out, **kw)
            want = _lib.compare_stats(ref, out)
            for k in ("mismatches", "first_index", "max_diff", "max_sq_error", "numel"):
                assert st[k] == want[k], (path, write_out, k, st[k], want[k])
            for k in ("sq_error_sum", "ref_sq_sum"):
                assert math.isclose(st[k], want[k], rel_tol=1e-12), (k, st[k], want[k])
            if o is not None:
                assert torch.equal(o.view(torch.int16) if o.dtype != torch.float32 else o.view(torch.int32),
                                   out.view(torch.int16) if out.dtype != torch.float32 else out.view(torch.int32))
    st, _ = _lib.gemm_compare(*t, out, **kw)
    assert st["mismatches"] == 0 and st["first_index"] == -1 and st["max_diff"] == 0


def test_suite_on_device_emul_vs_emul():
    """run_suite with the emulation as both sides (must match exactly) and the pseudo GEMM as the
    'real' side in MSE mode, on the GPU with the on-device comparison."""
    from emugen_b200 import suite
    from emugen_b200.backends.mxfp import build_mxfp_fns

    quant_fn, _real, emul_fn, pseudo_fn, _meta = build_mxfp_fns(return_pseudo=True)
    kw = dict(num_iterations=4, dims_m=[128, 256], dims_n=[64, 128], dims_k=[256, 512],
              distributions=["normal", "student_t", "outliers"], seed=3)
    assert suite.run_suite(quant_fn, emul_fn, emul_fn, **kw) == 0
    assert suite.run_suite(quant_fn, lambda s: pseudo_fn(s).to(torch.float16), emul_fn, metric_mode="mse", **kw) == 0


def test_fused_compare_returns_the_reference_mismatch_samples():
    """compare.gemm_compare_tensors: the comparison fused into the tensor-core epilogue (no output
    written) gives the same dict as compare_tensors on the full output -- status, max_diff and the
    first mismatch samples in row-major order, gathered from recomputed 128-row blocks (here across
    three blocks, with a NaN on the real side)."""
    from emugen_b200 import _lib, compare, nvfp4_global_scales, quant_nvfp4

    g = torch.Generator().manual_seed(31)
    a = torch.randn(512, 1024, generator=g).half().cuda()
    b = torch.randn(512, 1024, generator=g).half().cuda()
    gsa, gsb, alpha = nvfp4_global_scales(a, b)
    (qa, sa), (qb, sb) = quant_nvfp4(a, gsa), quant_nvfp4(b, gsb)
    # 512 x 512 x 1024 (2^28 MACs) takes the tensor-core path, whose epilogue does the comparison
    kw = dict(fmt=0, group_size=16, w_reduce=4, stage3_rounding=0, stage4_rounding=0, alpha=alpha, out_mode=0)
    out = _lib.gemm(qa, qb, sa, sb, **kw)

    def same(x, y):   # the two dicts equal, a NaN sample value equal to a NaN
        def norm(d):
            return [(e["idx"], "nan" if math.isnan(e["real"]) else e["real"], e["model"], e["diff"])
                    for e in d["mismatch_details"]]
        return x["status"] == y["status"] and x["max_diff"] == y["max_diff"] and norm(x) == norm(y)

    assert same(compare.gemm_compare_tensors(qa, qb, sa, sb, out.clone(), **kw), compare.compare_tensors(out, out))
    real = out.clone()
    for r, c in ((130, 5), (130, 7), (131, 0), (300, 10), (511, 511)):
        real[r, c] = real[r, c] + 1.0
    real[300, 11] = float("nan")
    for n in (1, 3, 5, 8):
        got = compare.gemm_compare_tensors(qa, qb, sa, sb, real, sample_count=n, **kw)
        assert same(got, compare.compare_tensors(real, out, sample_count=n))
        assert [d["idx"] for d in got["mismatch_details"]] == [(130, 5), (130, 7), (131, 0), (300, 10), (300, 11),
                                                               (511, 511)][:n]
