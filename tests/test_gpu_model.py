"""GPU: the accumulator-model GEMM (emu_gemm_model: alignment widths, aligned-addend rounding,
stage-3 order) against the C oracle's restatement of the same model, bit for bit.  The model has
no reference counterpart (the reference ignores w_stage3 / w_stage4); the all-zero model is the
reference model and must equal emu_gemm."""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden.make_golden import gen_inputs
from tests.golden_cases import nan_equal_mismatches

pytestmark = pytest.mark.gpu

MODELS = [(24, 0, 0, 0), (31, 0, 1, 0), (0, 24, 0, 0), (0, 28, 1, 0), (25, 31, 0, 0), (30, 24, 1, 0),
          (0, 0, 0, 1), (0, 0, 0, 2), (8, 12, 0, 0), (46, 52, 1, 0)]
CASES = []
for i, (kind, data) in enumerate([("nvfp", "normal"), ("nvfp", "outliers"), ("nvfp", "cancel"), ("nvfp", "raw"),
                                  ("mxfp", "student_t"), ("mxfp", "outliers"), ("mxfp", "raw_scales_full"),
                                  ("nvfp", "huge_scales")]):
    for wr in ([1, 2, 4, 8] if kind == "nvfp" else [1, 2, 4]):
        CASES.append((kind, data, wr, MODELS[(i * 3 + wr) % len(MODELS)], i % 3))


def _run(case_id, kind, data, wr, model, out_mode, K=512):
    from emugen_b200 import _lib

    M, N = 96, 80
    rng = np.random.default_rng(zlib.crc32(f"model-{case_id}".encode()))
    a, b, sfa, sfb, alpha = gen_inputs(dict(kind=kind, data=data, M=M, N=N, K=K), rng)
    al = float(alpha) if kind == "nvfp" else None
    gs = 16 if kind == "nvfp" else 32
    a3, a4, rm, order = model
    got = _lib.gemm_model(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(sfa).cuda(),
                          torch.from_numpy(sfb).cuda(), fmt=0 if kind == "nvfp" else 1, group_size=gs, w_reduce=wr,
                          stage3_rounding=0, stage4_rounding=1,
                          alpha=None if al is None else torch.tensor([al]), out_mode=out_mode,
                          align3=a3, align4=a4, align_rounding=rm, order=order)
    ref = oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0 if kind == "nvfp" else 1, group_size=gs, w_reduce=wr, r3=0,
                           r4=1, alpha=al, out_mode=out_mode, align3=a3, align4=a4, align_rm=rm, order=order)
    return got, ref


# w_reduce 3 (the general kernel), and K that ends inside a chunk (NVFP4 w_reduce 1, 2: K = 80, 160;
# MXFP4 w_reduce 4 with K = 384, three 128-element chunks)
EXTRA = [("nvfp", "normal", 3, (26, 30, 0, 0), 0, 528), ("nvfp", "outliers", 1, (24, 24, 1, 0), 1, 80),
         ("nvfp", "cancel", 2, (0, 0, 0, 2), 2, 160), ("mxfp", "student_t", 4, (27, 29, 1, 0), 0, 384),
         ("mxfp", "outliers", 3, (0, 0, 0, 1), 1, 384)]


@pytest.mark.parametrize("kind,data,wr,model,out_mode,K", EXTRA,
                         ids=[f"{c[0]}-{c[1]}-wr{c[2]}-K{c[5]}" for c in EXTRA])
def test_model_other_shapes(kind, data, wr, model, out_mode, K):
    got, ref = _run(f"x{kind}{data}{wr}{model}{K}", kind, data, wr, model, out_mode, K)
    if out_mode == 2:
        g = got.cpu().numpy()
        gn, rn = np.isnan(g), np.isnan(ref)
        assert np.array_equal(gn, rn) and np.array_equal(g[~gn].view(np.uint32), ref[~rn].view(np.uint32))
    else:
        bits = got.cpu().view(torch.int16).numpy().view(np.uint16)
        assert nan_equal_mismatches(bits, ref, "bfloat16" if out_mode == 1 else "float16") == 0


@pytest.mark.parametrize("kind,data,wr,model,out_mode", CASES,
                         ids=[f"{c[0]}-{c[1]}-wr{c[2]}-{'_'.join(map(str, c[3]))}" for c in CASES])
def test_model_matches_oracle(kind, data, wr, model, out_mode):
    got, ref = _run(f"{kind}{data}{wr}{model}", kind, data, wr, model, out_mode)
    if out_mode == 2:
        g = got.cpu().numpy()
        gn, rn = np.isnan(g), np.isnan(ref)
        assert np.array_equal(gn, rn) and np.array_equal(g[~gn].view(np.uint32), ref[~rn].view(np.uint32))
    else:
        bits = got.cpu().view(torch.int16).numpy().view(np.uint16)
        assert nan_equal_mismatches(bits, ref, "bfloat16" if out_mode == 1 else "float16") == 0


def test_model_changes_results_and_zero_model_is_reference():
    from emugen_b200 import _lib

    rng = np.random.default_rng(5)
    a, b, sfa, sfb, alpha = gen_inputs(dict(kind="nvfp", data="cancel", M=128, N=64, K=1024), rng)
    t = [torch.from_numpy(x).cuda() for x in (a, b, sfa, sfb)]
    kw = dict(fmt=0, group_size=16, w_reduce=4, stage3_rounding=0, stage4_rounding=0,
              alpha=torch.tensor([float(alpha)]), out_mode=2)
    base = _lib.gemm(*t, **kw)
    zero = _lib.gemm_model(*t, **kw)
    assert torch.equal(base.view(torch.int32), zero.view(torch.int32))
    narrow = _lib.gemm_model(*t, align3=8, align4=8, **kw)
    assert not torch.equal(base.view(torch.int32), narrow.view(torch.int32))
