"""GPU parity of the skinny-problem kernel (M < 128 with K a multiple of 64: decode shapes), bit for
bit against the C oracle, and its agreement with the general CUDA-core kernel."""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden.make_golden import gen_inputs
from tests.golden_cases import nan_equal_mismatches

pytestmark = pytest.mark.gpu

CASES = [
    # kind, data, M, N, K, w_reduce, r3, r4, out_mode
    ("nvfp", "normal", 1, 130, 512, 4, 0, 0, 0),
    ("nvfp", "outliers", 8, 200, 1024, 4, 1, 0, 1),
    ("nvfp", "raw_nan_scales", 5, 64, 256, 4, 0, 1, 0),
    ("nvfp", "cancel", 17, 33, 2048, 1, 1, 1, 2),
    ("nvfp", "huge_scales", 32, 96, 512, 16, 0, 0, 0),
    ("nvfp", "fp16_round", 64, 65, 128, 2, 0, 1, 1),
    ("nvfp", "abs_normal", 3, 1000, 4096, 4, 0, 0, 0),
    ("mxfp", "normal", 1, 300, 1024, 2, 0, 0, 0),
    ("mxfp", "student_t", 4, 129, 512, 2, 1, 0, 1),
    ("mxfp", "raw_scales_full", 16, 64, 256, 2, 0, 1, 2),
    ("mxfp", "subnormal_acc", 33, 80, 512, 1, 1, 1, 0),
    ("mxfp", "flt_max", 7, 70, 128, 2, 0, 0, 2),
    # one row of A (its own kernel, 4096-element K windows): several windows and a partial last one,
    # windows of 64 blocks (w_reduce 1, 2, 4) and of 16 blocks (w_reduce 16), a partial 32-column tile
    ("nvfp", "normal", 1, 170, 9216, 4, 0, 0, 0),
    ("nvfp", "outliers", 1, 70, 4160, 1, 1, 1, 2),
    ("nvfp", "cancel", 1, 64, 5120, 16, 0, 1, 0),
    ("nvfp", "raw_nan_scales", 1, 96, 4608, 4, 1, 1, 1),
    ("mxfp", "student_t", 1, 100, 8256, 2, 1, 0, 1),
    ("mxfp", "subnormal_acc", 1, 40, 6144, 1, 0, 0, 2),
]


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("kind,data,M,N,K,wr,r3,r4,out", CASES, ids=[f"{c[0]}-{c[1]}-{c[2]}x{c[3]}x{c[4]}-wr{c[5]}" for c in CASES])
def test_skinny_vs_oracle_and_general_kernel(kind, data, M, N, K, wr, r3, r4, out):
    from emugen_b200 import _lib

    rng = np.random.default_rng(zlib.crc32(f"skinny-{kind}-{data}-{M}-{N}-{K}".encode()))
    a, b, sfa, sfb, alpha = gen_inputs(dict(kind=kind, data=data, M=M, N=N, K=K), rng)
    gs = 16 if kind == "nvfp" else 32
    al = float(alpha) if kind == "nvfp" else None
    t = [torch.from_numpy(x).cuda() for x in (a, b, sfa, sfb)]
    kw = dict(fmt=0 if kind == "nvfp" else 1, group_size=gs, w_reduce=wr, stage3_rounding=r3, stage4_rounding=r4,
              alpha=None if al is None else torch.tensor([al], device="cuda"), out_mode=out)
    got = _lib.gemm(*t, path="simt", **kw)          # no workspace: M < 128 takes the skinny kernel
    general = _lib.gemm_model(*t, align3=0, align4=0, order=2, **kw) if wr <= 16 else None
    ref = oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0 if kind == "nvfp" else 1, group_size=gs, w_reduce=wr, r3=r3,
                           r4=r4, alpha=al, out_mode=out)
    if out == 2:
        g = got.cpu().numpy()
        gn, rn = np.isnan(g), np.isnan(ref)
        assert np.array_equal(gn, rn) and np.array_equal(g[~gn].view(np.uint32), ref[~rn].view(np.uint32))
    else:
        assert nan_equal_mismatches(_bits(got), ref, "bfloat16" if out == 1 else "float16") == 0
    del general


def test_decode_shape_timing_smoke():
    """The decode shapes of the benchmark configuration run: M = 1, 8, 32 x (N, K) =
    (128256, 4096), sampled columns checked against the oracle."""
    from emugen_b200 import _lib
    from tests.golden.make_golden import pad, swizzle

    rng = np.random.default_rng(77)
    N, K = 128256, 4096
    G = K // 16
    b = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    sb = rng.integers(0x30, 0x48, (N, G), dtype=np.uint8)
    sbz = swizzle(sb, pad(N, 128), pad(G, 4))
    tb, tsb = torch.from_numpy(b).cuda(), torch.from_numpy(sbz).cuda()
    for M in (1, 8, 32):
        a = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
        sa = rng.integers(0x30, 0x48, (M, G), dtype=np.uint8)
        saz = swizzle(sa, pad(M, 128), pad(G, 4))
        got = _lib.gemm(torch.from_numpy(a).cuda(), tb, torch.from_numpy(saz).cuda(), tsb, fmt=0, group_size=16,
                        w_reduce=4, stage3_rounding=0, stage4_rounding=0, alpha=None, out_mode=0)
        cols = rng.choice(N, 64, replace=False)
        ref = oracle.emul_gemm(a, b[cols], saz, swizzle(sb[cols], 128, pad(G, 4)), scale_fmt=0, group_size=16,
                               w_reduce=4, alpha=None, out_mode=0)
        assert nan_equal_mismatches(_bits(got)[:, cols], ref, "float16") == 0


@pytest.mark.parametrize("kind", ["nvfp", "mxfp"])
@pytest.mark.parametrize("M,N", [(0, 64), (64, 0), (0, 0), (1, 1)])
def test_degenerate_shapes(kind, M, N):
    """Empty and single-output problems through the C ABI: an empty output is returned without a launch
    failure, a 1x1 output matches the oracle."""
    from emugen_b200 import _lib
    from tests.golden.make_golden import pad, swizzle

    K = 128
    gs = 16 if kind == "nvfp" else 32
    G = K // gs
    rng = np.random.default_rng(M * 131 + N + (7 if kind == "mxfp" else 0))
    a = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
    b = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    if kind == "nvfp":
        sa = rng.integers(0x20, 0x50, size=(max(M, 1), G), dtype=np.uint8)
        sb = rng.integers(0x20, 0x50, size=(max(N, 1), G), dtype=np.uint8)
    else:
        sa = rng.integers(120, 135, size=(max(M, 1), G), dtype=np.uint8)
        sb = rng.integers(120, 135, size=(max(N, 1), G), dtype=np.uint8)
    sfa = swizzle(sa, pad(max(M, 1), 128), pad(G, 4))
    sfb = swizzle(sb, pad(max(N, 1), 128), pad(G, 4))
    alpha = 0.5 if kind == "nvfp" else None
    al = None if alpha is None else torch.tensor([alpha], dtype=torch.float32, device="cuda")
    got = _lib.gemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(sfa).cuda(),
                    torch.from_numpy(sfb).cuda(), fmt=0 if kind == "nvfp" else 1, group_size=gs,
                    w_reduce=4 if kind == "nvfp" else 2, stage3_rounding=0, stage4_rounding=0, alpha=al, out_mode=0)
    torch.cuda.synchronize()
    assert tuple(got.shape) == (M, N)
    if M and N:
        ref = oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0 if kind == "nvfp" else 1, group_size=gs,
                               w_reduce=4 if kind == "nvfp" else 2, alpha=alpha, out_mode=0)
        assert nan_equal_mismatches(_bits(got), ref, "float16") == 0
