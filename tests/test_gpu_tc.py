"""GPU parity of the tensor-core (tcgen05) path: every input distribution of the golden set,
regenerated at shapes that take the tensor-core kernel (M >= 128, N >= 64, K % 64 == 0), compared bit
for bit (NaN payloads excepted) with the C oracle and with the CUDA-core kernel."""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden.make_golden import gen_inputs
from tests.golden_cases import nan_equal_mismatches

pytestmark = pytest.mark.gpu

NV_DATA = ["normal", "abs_normal", "outliers", "mixed_rows", "cancel", "raw", "raw_nan_scales", "all_neg_zero",
           "fp16_round", "huge_scales", "tiny_scales"]
MX_DATA = ["normal", "student_t", "abs_normal", "outliers", "cancel", "raw_scales_full", "subnormal_acc", "flt_max",
           "fp16_round", "all_neg_zero", "huge_bf16"]

CASES = []
for i, d in enumerate(NV_DATA):
    CASES.append(dict(kind="nvfp", data=d, M=[128, 200, 256][i % 3], N=[64, 100, 192][(i + 1) % 3],
                      K=[256, 512, 64, 1024][i % 4], r3=i % 2, r4=(i // 2) % 2, out=i % 3))
for i, d in enumerate(MX_DATA):
    CASES.append(dict(kind="mxfp", data=d, M=[128, 200, 256][i % 3], N=[64, 100, 192][(i + 1) % 3],
                      K=[256, 512, 64, 1024][i % 4] if d != "flt_max" else 128, r3=i % 2, r4=(i // 2) % 2,
                      out=i % 3))
CASES.append(dict(kind="nvfp", data="abs_normal", M=512, N=320, K=4096, r3=0, r4=0, out=0))
CASES.append(dict(kind="mxfp", data="normal", M=384, N=256, K=4096, r3=1, r4=0, out=1))


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _run(a, b, sfa, sfb, kind, r3, r4, alpha, out_mode, path):
    from emugen_b200 import _lib

    dev = "cuda"
    al = None if alpha is None else torch.tensor([alpha], dtype=torch.float32, device=dev)
    return _lib.gemm(torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev), torch.from_numpy(sfa).to(dev),
                     torch.from_numpy(sfb).to(dev), fmt=0 if kind == "nvfp" else 1,
                     group_size=16 if kind == "nvfp" else 32, w_reduce=4 if kind == "nvfp" else 2,
                     stage3_rounding=r3, stage4_rounding=r4, alpha=al, out_mode=out_mode, path=path)


def _compare(got, ref, out_mode):
    if out_mode == 2:
        g = got.cpu().numpy()
        gn, rn = np.isnan(g), np.isnan(ref)
        return int((gn != rn).sum() + (g[~gn & ~rn].view(np.uint32) != ref[~gn & ~rn].view(np.uint32)).sum())
    return nan_equal_mismatches(_bits(got), ref, "bfloat16" if out_mode == 1 else "float16")


@pytest.mark.parametrize("case", CASES, ids=[f"{c['kind']}-{c['data']}-{c['M']}x{c['N']}x{c['K']}" for c in CASES])
def test_tc_vs_oracle_and_simt(case):
    from emugen_b200 import _lib

    rng = np.random.default_rng(zlib.crc32(f"{case['kind']}-{case['data']}-{case['M']}-{case['K']}".encode()))
    a, b, sfa, sfb, alpha = gen_inputs(case, rng)
    kind = case["kind"]
    alpha = float(alpha) if kind == "nvfp" else None
    params = _lib.EmuGemmParams(0 if kind == "nvfp" else 1, 16 if kind == "nvfp" else 32, 4 if kind == "nvfp" else 2,
                                case["r3"], case["r4"], case["out"])
    import ctypes

    assert _lib.load().emu_gemm_tc_workspace_size(case["M"], case["N"], case["K"], ctypes.byref(params)) > 0
    got = _run(a, b, sfa, sfb, kind, case["r3"], case["r4"], alpha, case["out"], "tc")
    simt = _run(a, b, sfa, sfb, kind, case["r3"], case["r4"], alpha, case["out"], "simt")
    ref = oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0 if kind == "nvfp" else 1, group_size=16 if kind == "nvfp" else 32,
                           w_reduce=4 if kind == "nvfp" else 2, r3=case["r3"], r4=case["r4"], alpha=alpha,
                           out_mode=case["out"])
    assert _compare(got, ref, case["out"]) == 0
    assert _compare(simt, ref, case["out"]) == 0


def test_tc_8192_sampled_against_oracle():
    """The benchmark shape (8192^3 NVFP4, |N(0,1)| + outlier columns, quantised by libemugen): full
    tensor-core launch, 64 sampled outputs re-derived by the oracle on row / column slices, in fp16 (the
    emulator's output, saturated at this data) and in the f32 output mode (the accumulator)."""
    from emugen_b200 import nvfp4_global_scales, quant_nvfp4
    from tests.golden.make_golden import pad, swizzle

    g = torch.Generator().manual_seed(3)
    M = N = K = 8192
    xa = torch.randn(M, K, generator=g).abs_()
    xb = torch.randn(N, K, generator=g).abs_()
    cols = torch.randperm(K, generator=g)[:82]
    xa[:, cols] *= 100
    xb[:, cols] *= 100
    xa, xb = xa.half().cuda(), xb.half().cuda()
    gsa, gsb, alpha = nvfp4_global_scales(xa, xb)
    qa, sfa = quant_nvfp4(xa, gsa)
    qb, sfb = quant_nvfp4(xb, gsb)
    a, b, sfa, sfb = qa.cpu().numpy(), qb.cpu().numpy(), sfa.cpu().numpy(), sfb.cpu().numpy()
    al = float(alpha.item())
    got = _bits(_run(a, b, sfa, sfb, "nvfp", 0, 0, al, 0, "tc"))
    # f32 output mode: the accumulator itself (|C| ~ 5e5 here, so the fp16 output is +inf everywhere)
    got32 = _run(a, b, sfa, sfb, "nvfp", 0, 0, al, 2, "tc").cpu().numpy()
    rng = np.random.default_rng(5)
    rows = rng.choice(M, 8, replace=False)
    cs = rng.choice(N, 8, replace=False)
    G = K // 16

    def lin(sf, idx):
        flat = sf.reshape(-1)
        out = np.empty((len(idx), G), dtype=np.uint8)
        for i, r in enumerate(idx):
            out[i] = [flat[oracle.swizzle_offset(int(r), c, sf.shape[1])] for c in range(G)]
        return swizzle(out, 128, pad(G, 4))

    ref = oracle.emul_gemm(a[rows], b[cs], lin(sfa, rows), lin(sfb, cs), scale_fmt=0, group_size=16, w_reduce=4,
                           alpha=al, out_mode=0)
    assert nan_equal_mismatches(got[np.ix_(rows, cs)], ref, "float16") == 0
    ref32 = oracle.emul_gemm(a[rows], b[cs], lin(sfa, rows), lin(sfb, cs), scale_fmt=0, group_size=16, w_reduce=4,
                             alpha=al, out_mode=2)
    g32 = np.ascontiguousarray(got32[np.ix_(rows, cs)])
    assert np.isfinite(g32).all() and np.abs(g32).min() > 65504
    assert (g32.view(np.uint32) != np.ascontiguousarray(ref32).view(np.uint32)).sum() == 0


def test_tc_mxfp4_8192_sampled_against_oracle():
    """MXFP4 at 8192^3 (bf16 ~N(0,1) inputs, quantised by libemugen): the f32 block-sum launch at full
    size.  64 sampled outputs re-derived by the oracle on row / column slices, in
    the f32 output mode (the accumulator) and in bf16 (fp16 then bf16, the reference's output path)."""
    from emugen_b200 import quant_mxfp4
    from tests.golden.make_golden import pad, swizzle

    g = torch.Generator().manual_seed(11)
    M = N = K = 8192
    xa = torch.randn(M, K, generator=g).bfloat16().cuda()
    xb = torch.randn(N, K, generator=g).bfloat16().cuda()
    qa, sfa = quant_mxfp4(xa)
    qb, sfb = quant_mxfp4(xb)
    a, b, sfa, sfb = qa.cpu().numpy(), qb.cpu().numpy(), sfa.cpu().numpy(), sfb.cpu().numpy()
    got32 = _run(a, b, sfa, sfb, "mxfp", 0, 0, None, 2, "tc").cpu().numpy()
    got16 = _bits(_run(a, b, sfa, sfb, "mxfp", 0, 0, None, 1, "tc"))
    rng = np.random.default_rng(6)
    rows = rng.choice(M, 8, replace=False)
    cs = rng.choice(N, 8, replace=False)
    G = K // 32

    def lin(sf, idx):
        flat = sf.reshape(-1)
        out = np.empty((len(idx), G), dtype=np.uint8)
        for i, r in enumerate(idx):
            out[i] = [flat[oracle.swizzle_offset(int(r), c, pad(G, 4))] for c in range(G)]
        return swizzle(out, 128, pad(G, 4))

    la, lb = lin(sfa, rows), lin(sfb, cs)
    ref32 = oracle.emul_gemm(a[rows], b[cs], la, lb, scale_fmt=1, group_size=32, w_reduce=2, out_mode=2)
    g32 = np.ascontiguousarray(got32[np.ix_(rows, cs)])
    assert np.isfinite(g32).all()
    assert (g32.view(np.uint32) != np.ascontiguousarray(ref32).view(np.uint32)).sum() == 0
    ref16 = oracle.emul_gemm(a[rows], b[cs], la, lb, scale_fmt=1, group_size=32, w_reduce=2, out_mode=1)
    assert nan_equal_mismatches(got16[np.ix_(rows, cs)], ref16, "bfloat16") == 0


OUTLIER_CASES = [("nvfp", True, 0, 0, 0, 100.0), ("nvfp", False, 1, 1, 1, 100.0), ("nvfp", True, 1, 0, 2, 1000.0),
                 ("nvfp", False, 0, 1, 0, 30.0), ("mxfp", True, 0, 0, 1, 1000.0), ("mxfp", False, 1, 1, 0, 1e4),
                 # shrunken channels: finer quanta than the rest, so the exactness bound of the f32
                 # accumulator update decides per tile pair (RZ) while RNE always takes it
                 ("nvfp", False, 0, 0, 0, 1e-3), ("nvfp", True, 1, 1, 1, 1e-3), ("mxfp", False, 0, 0, 0, 1e-6),
                 ("mxfp", True, 1, 1, 2, 1e-9)]


@pytest.mark.parametrize("kind,absval,r3,r4,out,factor", OUTLIER_CASES,
                         ids=[f"{k}-{'abs' if a else 'signed'}-r{r3}{r4}-o{o}-x{f:g}" for k, a, r3, r4, o, f in OUTLIER_CASES])
def test_tc_outlier_channels(kind, absval, r3, r4, out, factor):
    """The benchmark's input recipe at 256x192x4096: 1% of the K channels scaled in both A and B, so
    the K blocks holding one of them carry a group whose scales dwarf the others' and leave the
    block-sum path (mixed path: the other groups' block sum plus one separate group; integer path
    otherwise).  Quantised on the device, compared bit for bit with the oracle and the CUDA-core kernel."""
    from emugen_b200 import nvfp4_global_scales, quant_mxfp4, quant_nvfp4

    g = torch.Generator().manual_seed(int(factor) + 7 * r3 + 3 * r4 + (11 if absval else 0) + (5 if factor < 1 else 0))
    M, N, K = 256, 192, 4096
    xa, xb = torch.randn(M, K, generator=g), torch.randn(N, K, generator=g)
    if absval:
        xa, xb = xa.abs_(), xb.abs_()
    cols = torch.randperm(K, generator=g)[:K // 100]
    xa[:, cols] *= factor
    xb[:, cols] *= factor
    xa, xb = xa.half().cuda(), xb.half().cuda()
    if kind == "nvfp":
        gsa, gsb, al = nvfp4_global_scales(xa, xb)
        (qa, sfa), (qb, sfb) = quant_nvfp4(xa, gsa), quant_nvfp4(xb, gsb)
        alpha = float(al.item())
    else:
        (qa, sfa), (qb, sfb) = quant_mxfp4(xa), quant_mxfp4(xb)
        alpha = None
    a, b, sfa, sfb = qa.cpu().numpy(), qb.cpu().numpy(), sfa.cpu().numpy(), sfb.cpu().numpy()
    got = _run(a, b, sfa, sfb, kind, r3, r4, alpha, out, "tc")
    simt = _run(a, b, sfa, sfb, kind, r3, r4, alpha, out, "simt")
    ref = oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0 if kind == "nvfp" else 1, group_size=16 if kind == "nvfp" else 32,
                           w_reduce=4 if kind == "nvfp" else 2, r3=r3, r4=r4, alpha=alpha, out_mode=out)
    assert _compare(simt, ref, out) == 0
    assert _compare(got, ref, out) == 0


@pytest.mark.parametrize("r4", [0, 1])
def test_tc_split_launches(r4):
    """One call whose tile pairs go to both launches: outlier channels in the first 128 rows of A and
    the first 64 rows of B only, so tile pairs touching either keep most blocks off the block-sum path
    (f64 launch) while the others stay on it (f32 launch).  Compared bit for bit with the oracle."""
    from emugen_b200 import nvfp4_global_scales, quant_nvfp4

    g = torch.Generator().manual_seed(101 + r4)
    M, N, K = 256, 256, 4096
    xa, xb = torch.randn(M, K, generator=g), torch.randn(N, K, generator=g)
    cols = torch.randperm(K, generator=g)[:K // 50]
    xa[:128, cols] *= 100
    xb[:64, cols] *= 100
    xa, xb = xa.half().cuda(), xb.half().cuda()
    gsa, gsb, al = nvfp4_global_scales(xa, xb)
    (qa, sfa), (qb, sfb) = quant_nvfp4(xa, gsa), quant_nvfp4(xb, gsb)
    alpha = float(al.item())
    a, b, sfa, sfb = qa.cpu().numpy(), qb.cpu().numpy(), sfa.cpu().numpy(), sfb.cpu().numpy()
    got = _run(a, b, sfa, sfb, "nvfp", 0, r4, alpha, 0, "tc")
    ref = oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0, group_size=16, w_reduce=4, r3=0, r4=r4, alpha=alpha, out_mode=0)
    assert _compare(got, ref, 0) == 0
