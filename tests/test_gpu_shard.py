"""The one-GEMM split over ranks, on one GPU: the shards' amax words combined by MAX give the global
scales of the whole operand (gemm_compare/backends/nvfp.py:24-27), and the column slices (or the tiles
of a grid split) computed from each rank's rows of A and B, put in place, are the whole GEMM's output
bit for bit."""
import pytest
import torch

from emugen_b200 import shard

pytestmark = pytest.mark.gpu


def _inputs(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).abs_()
    b = torch.randn(n, k, generator=g).abs_()
    cols = torch.randperm(k, generator=g)[: max(1, k // 100)]
    a[:, cols] *= 100.0
    b[:, cols] *= 100.0
    return a.half().cuda(), b.half().cuda()


@pytest.mark.parametrize("world", [2, 3, 8])
def test_sharded_scales_and_column_split_equal_the_whole_gemm(world):
    from emugen_b200 import _lib

    M, N, K = 256, 1000, 1024
    a, b = _inputs(M, N, K, 5 + world)
    gsa, gsb, alpha = _lib.nvfp4_global_scales(a, b)
    ranges = [shard.column_range(N, world, r) for r in range(world)]
    words = [_lib.nvfp4_amax(a, b[n0:n1]) if n1 > n0 else None for n0, n1 in ranges]
    combined = torch.stack([w for w in words if w is not None]).max(dim=0).values
    sgsa, sgsb, salpha = _lib.nvfp4_scales_from_amax(combined)
    assert torch.equal(gsa, sgsa) and torch.equal(gsb, sgsb) and torch.equal(alpha, salpha)

    qa, sa = _lib.quant_nvfp4(a, gsa)
    qb, sb = _lib.quant_nvfp4(b, gsb)
    kw = dict(fmt=0, group_size=16, w_reduce=4, stage3_rounding=0, stage4_rounding=0, alpha=alpha, out_mode=2)
    whole = _lib.gemm(qa, qb, sa, sb, path="tc", **kw)
    parts = []
    for n0, n1 in ranges:
        if n1 == n0:
            continue
        # a rank quantises only its own rows of B, with the global scale of all of B
        qbs, sbs = _lib.quant_nvfp4(b[n0:n1], gsb)
        bq, bs = shard.b_slice(qb, sb, n0, n1)
        assert torch.equal(qbs, bq) and torch.equal(sbs, bs)
        parts.append(_lib.gemm(qa, qbs, sa, sbs, **kw))
    assert torch.equal(torch.cat(parts, dim=1).view(torch.int32), whole.view(torch.int32))


def test_sharded_amax_keeps_nan_and_zero_rules():
    """A NaN in one shard makes the combined amax NaN, which counts as amax 1.0 (global scale 2688, as
    for the whole operand); all-zero shards do not lower it."""
    from emugen_b200 import _lib

    a, b = _inputs(128, 256, 256, 1)
    b[200, 3] = float("nan")
    z = torch.zeros_like(b[:128])
    words = torch.stack([_lib.nvfp4_amax(a, b[:128]), _lib.nvfp4_amax(a, b[128:]), _lib.nvfp4_amax(a, z)])
    got = _lib.nvfp4_scales_from_amax(words.max(dim=0).values)
    want = _lib.nvfp4_global_scales(a, b)
    assert all(torch.equal(x, y) for x, y in zip(got, want))
    assert float(want[1]) == 2688.0


@pytest.mark.parametrize("world", [4, 8])
def test_grid_tiles_equal_the_whole_gemm(world):
    """A pr x pc grid (shard.grid_shape): rank tiles from rows of A and of B, both operands sharded, their
    global scales from the MAX of all ranks' amax words."""
    from emugen_b200 import _lib

    M, N, K = 384, 1000, 1024
    a, b = _inputs(M, N, K, 20 + world)
    gsa, gsb, alpha = _lib.nvfp4_global_scales(a, b)
    tiles = [shard.tile_ranges(M, N, world, r) for r in range(world)]
    words = torch.stack([_lib.nvfp4_amax(a[m0:m1], b[n0:n1]) for (m0, m1), (n0, n1) in tiles])
    sgsa, sgsb, salpha = _lib.nvfp4_scales_from_amax(words.max(dim=0).values)
    assert torch.equal(gsa, sgsa) and torch.equal(gsb, sgsb) and torch.equal(alpha, salpha)
    kw = dict(fmt=0, group_size=16, w_reduce=4, stage3_rounding=0, stage4_rounding=0, alpha=alpha, out_mode=2)
    (qa, sa), (qb, sb) = _lib.quant_nvfp4(a, gsa), _lib.quant_nvfp4(b, gsb)
    whole = _lib.gemm(qa, qb, sa, sb, path="tc", **kw)
    full = torch.empty_like(whole)
    for (m0, m1), (n0, n1) in tiles:
        qat, sat = _lib.quant_nvfp4(a[m0:m1], gsa)
        qbt, sbt = _lib.quant_nvfp4(b[n0:n1], gsb)
        ref_a, ref_sa = shard.row_slice(qa, sa, m0, m1)
        assert torch.equal(qat, ref_a) and torch.equal(sat, ref_sa)
        full[m0:m1, n0:n1] = _lib.gemm(qat, qbt, sat, sbt, **kw)
    assert torch.equal(full.view(torch.int32), whole.view(torch.int32))
