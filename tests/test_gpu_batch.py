"""emu_gemm_batch on the GPU: each parameter set's output equals emu_gemm_ws's under the same parameters
bit for bit, and each set's comparison with a reference equals emu_compare's on that set's output -- on
the tensor-core path (with the outputs, and fused into the epilogue without them) and on the CUDA-core
path, for NVFP4 and MXFP4."""
import pytest
import torch

pytestmark = pytest.mark.gpu

KEYS = ("mismatches", "first_index", "max_diff", "max_sq_error", "numel")


def _case(fmt, S, K, seed):
    from emugen_b200 import nvfp4_global_scales, quant_mxfp4, quant_nvfp4

    # columns spread over many binades (the MXFP4 sets' settings then change some outputs)
    g = torch.Generator().manual_seed(seed)
    spread = torch.exp(3.0 * torch.randn(1, K, generator=g))
    a = (torch.randn(S, K, generator=g) * spread).cuda()
    b = (torch.randn(S, K, generator=g) * spread).cuda()
    if fmt == 0:
        a, b = a.half(), b.half()
        gsa, gsb, alpha = nvfp4_global_scales(a, b)
        (qa, sa), (qb, sb) = quant_nvfp4(a, gsa), quant_nvfp4(b, gsb)
        return qa, qb, sa, sb, alpha
    (qa, sa), (qb, sb) = quant_mxfp4(a.bfloat16()), quant_mxfp4(b.bfloat16())
    return qa, qb, sa, sb, None


@pytest.mark.parametrize("fmt,S,K", [(0, 512, 1024), (0, 96, 256), (1, 512, 1024)])
def test_batch_equals_single_calls(fmt, S, K):
    from emugen_b200 import _lib

    qa, qb, sa, sb, alpha = _case(fmt, S, K, 5 + fmt + S)
    gs = 16 if fmt == 0 else 32
    blocks = (4, 2, 1, 8) if fmt == 0 else (2, 1, 4)
    sets = [(fmt, gs, wr, r3, r4, 2) for wr in blocks for r3, r4 in ((0, 0), (1, 1), (0, 1))]
    singles = [_lib.gemm(qa, qb, sa, sb, fmt=f, group_size=g, w_reduce=wr, stage3_rounding=r3, stage4_rounding=r4,
                         alpha=alpha, out_mode=om) for f, g, wr, r3, r4, om in sets]
    outs, stats = _lib.gemm_batch(qa, qb, sa, sb, sets, alpha=alpha)
    assert stats is None and outs.shape == (len(sets), S, S)
    for o, ref in zip(outs, singles):
        assert torch.equal(o.view(torch.int32), ref.view(torch.int32))

    # a reference that differs from every set's output somewhere (every 97th element of set 0's output
    # changed), so that each set's statistics -- count, first index, max diff -- are exercised
    ref = singles[0].clone()
    ref.view(-1)[::97] += 1.0
    outs, stats = _lib.gemm_batch(qa, qb, sa, sb, sets, alpha=alpha, ref=ref)
    for st, single in zip(stats, singles):
        want = _lib.compare_stats(ref, single)
        assert want["mismatches"] > 0 and all(st[k] == want[k] for k in KEYS), (st, want)
    if S >= 512:
        # no outputs: the comparisons fused into the tensor-core epilogue (its workspace whatever the size),
        # for the sets that path takes (block size 4 groups NVFP4, 2 MXFP4; the others run on the CUDA
        # cores, which need `out`)
        tc = [i for i, p in enumerate(sets) if p[2] == (4 if fmt == 0 else 2)]
        outs, stats = _lib.gemm_batch(qa, qb, sa, sb, [sets[i] for i in tc], alpha=alpha, ref=ref, write_out=False,
                                      path="tc")
        assert outs is None
        for st, i in zip(stats, tc):
            want = _lib.compare_stats(ref, singles[i])
            assert all(st[k] == want[k] for k in KEYS), (st, want)
