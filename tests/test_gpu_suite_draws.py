"""The reference's randomised suite, drawn the way its runner draws it (gemm_compare/runner.py:201-229:
M, N from {128, 256, 1024, 2048, 4096}, K from {128, 256, 512, 1024}, each operand from the six
default distributions of gemm_compare/data.py), run through this package's quant_fn + emul_fn and
compared in full with the C oracle: zero mismatches (NaN payloads aside), NVFP4 and MXFP4, 16 seeded
draws each."""
import random

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden_cases import nan_equal_mismatches

pytestmark = pytest.mark.gpu

DIMS_MN = [128, 256, 1024, 2048, 4096]
DIMS_K = [128, 256, 512, 1024]
DISTRIBUTIONS = ["normal", "uniform", "large", "outliers", "mixed_rows", "abs_large"]


def draws(n: int, seed: int):
    r = random.Random(seed)
    return [(r.choice(DIMS_MN), r.choice(DIMS_MN), r.choice(DIMS_K), r.choice(DISTRIBUTIONS), r.choice(DISTRIBUTIONS))
            for _ in range(n)]


@pytest.mark.parametrize("kind", ["nvfp", "mxfp"])
def test_suite_draws_match_the_oracle(kind):
    from emugen_b200.backends.mxfp import build_mxfp_fns
    from emugen_b200.backends.nvfp import build_nvfp_fns
    from emugen_b200.suite import DataGenerator

    nv = kind == "nvfp"
    dtype = torch.float16 if nv else torch.bfloat16
    quant_fn, _real, emul_fn, _meta = build_nvfp_fns() if nv else build_mxfp_fns(out_dtype=torch.bfloat16)
    bad = []
    for i, (M, N, K, da, db) in enumerate(draws(16, 7 if nv else 8)):
        g = torch.Generator().manual_seed(1000 * i + (1 if nv else 2))
        a = DataGenerator.get_random_tensor((M, K), da, device="cuda", dtype=dtype, generator=g)
        b = DataGenerator.get_random_tensor((N, K), db, device="cuda", dtype=dtype, generator=g)
        st = quant_fn(a, b)
        out = emul_fn(st)
        got = out.cpu().view(torch.int16).numpy().view(np.uint16)
        if nv:
            ref = oracle.emul_gemm(st.a_fp4.cpu().numpy(), st.b_fp4.cpu().numpy(),
                                   st.scale_a.view(torch.uint8).cpu().numpy(), st.scale_b.view(torch.uint8).cpu().numpy(),
                                   scale_fmt=0, group_size=16, w_reduce=4, alpha=float(st.alpha.item()))
            n_bad = nan_equal_mismatches(got, ref, "float16")
        else:
            ref = oracle.emul_gemm(st.a_fp4.cpu().numpy(), st.b_fp4.cpu().numpy(), st.a_scale.cpu().numpy(),
                                   st.b_scale.cpu().numpy(), scale_fmt=1, group_size=32, w_reduce=2,
                                   out_mode=oracle.OUT_BF16_VIA_F16)
            n_bad = nan_equal_mismatches(got, ref, "bfloat16")
        if n_bad:
            bad.append((i, M, N, K, da, db, n_bad))
    assert not bad, bad
