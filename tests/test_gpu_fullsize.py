"""Parity at the benchmarked sizes, in full rather than by sample.

* NVFP4 8192^3 on the benchmark's own data (|N(0,1)| fp16 with 1% of the K columns x100, seeded as
  bench.py draws it): every output of the tensor-core kernel against the CUDA-core kernel on the
  device, in the f32 output mode (the accumulator: the fp16 output saturates to inf at this data),
  and complete 128 x 64 output tiles against the C oracle, at least one per epilogue path class the
  kernel chose (read from its path codes), plus a whole 128-row band.
* NVFP4 8192^3 on |N(0,1)| without outlier channels (no saturation: block-sum path, f32 launch):
  every output against the CUDA-core kernel and a whole 128-row band against the oracle, in fp16.
* MXFP4 4096^3, the C2 configuration (bf16 in, bf16 out): two ~N(0,1) and two Student-t(3) cases,
  every output against the oracle.
Bar: bit-exact, NaN payloads aside (reference compare rule, gemm_compare/runner.py:20-32).
Reference: nvfp_emulation.cpp:90-156, mxfp_emulation.cpp:98-166, search/emulation/gemm.py:69.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden_cases import nan_equal_mismatches

pytestmark = pytest.mark.gpu

S = 8192
BM, BN, BK = 128, 64, 64


def _c3_inputs(outliers: bool, seed: int = 1234):
    """bench.py's make_inputs(0) (outliers=True), or the same draw without the outlier channels."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(S, S, generator=g).abs_()
    b = torch.randn(S, S, generator=g).abs_()
    cols = torch.randperm(S, generator=g)[: int(round(S * 0.01))]
    if outliers:
        a[:, cols] *= 100.0
        b[:, cols] *= 100.0
    return a.half().cuda(), b.half().cuda()


def _quant_nvfp4(a, b):
    from emugen_b200 import nvfp4_global_scales, quant_nvfp4

    gsa, gsb, alpha = nvfp4_global_scales(a, b)
    (qa, sa), (qb, sb) = quant_nvfp4(a, gsa), quant_nvfp4(b, gsb)
    return qa, qb, sa, sb, alpha


def _gemm_tc_with_paths(qa, qb, sa, sb, alpha, fmt, out_mode, r=0):
    """The tensor-core path through emu_gemm_ws with a workspace of our own, so that the kernel's
    per-block path codes can be read back: (output, codes [tiles_m, tiles_n, K/64])."""
    from emugen_b200 import _lib

    L = _lib.load()
    M, N, K = qa.shape[0], qb.shape[0], qa.shape[1] * 2
    prm = _lib.EmuGemmParams(fmt, 16 if fmt == 0 else 32, 4 if fmt == 0 else 2, r, r, out_mode)
    need = L.emu_gemm_tc_workspace_size(M, N, K, ctypes.byref(prm))
    off = L.emu_gemm_tc_path_offset(M, N, K, ctypes.byref(prm))
    assert need > 0 and off < need
    ws = torch.empty(need + 1024, dtype=torch.uint8, device="cuda")
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    odt = {0: torch.float16, 1: torch.bfloat16, 2: torch.float32}[out_mode]
    out = torch.empty((M, N), dtype=odt, device="cuda")
    st = L.emu_gemm_ws(qa.data_ptr(), qb.data_ptr(), sa.data_ptr(), sb.data_ptr(), M, N, K, sa.shape[0], sa.shape[1],
                       sb.shape[0], sb.shape[1], None if alpha is None else alpha.data_ptr(), ctypes.byref(prm),
                       out.data_ptr(), base, need, torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.emu_last_error().decode()
    _lib.device_status()
    tm, tn, nb = (M + BM - 1) // BM, (N + BN - 1) // BN, K // BK
    start = base - ws.data_ptr() + off
    codes = ws[start:start + tm * tn * nb].cpu().numpy().reshape(tm, tn, nb)
    return out, codes


def _simt(qa, qb, sa, sb, alpha, fmt, out_mode, r=0):
    from emugen_b200 import _lib

    return _lib.gemm(qa, qb, sa, sb, fmt=fmt, group_size=16 if fmt == 0 else 32, w_reduce=4 if fmt == 0 else 2,
                     stage3_rounding=r, stage4_rounding=r, alpha=alpha, out_mode=out_mode, path="simt")


def _oracle_block(a, b, sfa, sfb, rows0, nrows, cols0, ncols, fmt, alpha, out_mode):
    """Oracle outputs [rows0, +nrows) x [cols0, +ncols) from whole 128-row scale blocks (the swizzled
    layout keeps each 128-row block contiguous)."""
    r0, c0 = rows0 // 128 * 128, cols0 // 128 * 128
    r1, c1 = min(a.shape[0], -(-(rows0 + nrows) // 128) * 128), min(b.shape[0], -(-(cols0 + ncols) // 128) * 128)
    ref = oracle.emul_gemm(a[r0:r1], b[c0:c1], sfa[r0:r0 + -(-(r1 - r0) // 128) * 128],
                           sfb[c0:c0 + -(-(c1 - c0) // 128) * 128], scale_fmt=fmt, group_size=16 if fmt == 0 else 32,
                           w_reduce=4 if fmt == 0 else 2, alpha=alpha, out_mode=out_mode)
    return ref[rows0 - r0:rows0 - r0 + nrows, cols0 - c0:cols0 - c0 + ncols]


def _f32_mismatches(got: np.ndarray, ref: np.ndarray) -> int:
    gn, rn = np.isnan(got), np.isnan(ref)
    return int((gn != rn).sum() + (got[~gn & ~rn].view(np.uint32) != ref[~gn & ~rn].view(np.uint32)).sum())


def test_c3_benchmark_data_every_output_and_whole_tiles_per_path_class():
    from emugen_b200 import _lib

    qa, qb, sa, sb, alpha = _quant_nvfp4(*_c3_inputs(outliers=True))
    out, codes = _gemm_tc_with_paths(qa, qb, sa, sb, alpha, 0, 2)
    simt = _simt(qa, qb, sa, sb, alpha, 0, 2)
    st = _lib.compare_stats(simt, out)
    assert st["mismatches"] == 0, st
    got = out.cpu().numpy()
    assert np.isfinite(got).all() and np.abs(got).min() > 65504   # the f32 accumulator, beyond fp16's range
    a, b, sfa, sfb = (x.cpu().numpy() for x in (qa, qb, sa.view(torch.uint8), sb.view(torch.uint8)))
    al = float(alpha.item())
    cls = codes & 3
    present = [c for c in range(4) if (cls == c).any()]
    assert {1, 2, 3} <= set(present), present          # integer, block-sum and mixed blocks all occur
    tiles = set()
    for c in present:                                   # the tile pair with the most blocks of each class
        tiles.add(np.unravel_index(int(np.argmax((cls == c).sum(-1))), cls.shape[:2]))
    for tm, tn in sorted(tiles):
        ref = _oracle_block(a, b, sfa, sfb, tm * BM, BM, tn * BN, BN, 0, al, 2)
        assert _f32_mismatches(np.ascontiguousarray(got[tm * BM:(tm + 1) * BM, tn * BN:(tn + 1) * BN]), ref) == 0, (tm, tn)
    band = 37                                           # a whole 128-row band: every column tile
    ref = _oracle_block(a, b, sfa, sfb, band * BM, BM, 0, S, 0, al, 2)
    assert _f32_mismatches(np.ascontiguousarray(got[band * BM:(band + 1) * BM]), ref) == 0


def test_nvfp4_8192_without_outliers_fp16_every_output_and_a_band():
    from emugen_b200 import _lib

    qa, qb, sa, sb, alpha = _quant_nvfp4(*_c3_inputs(outliers=False, seed=99))
    out, codes = _gemm_tc_with_paths(qa, qb, sa, sb, alpha, 0, 0)
    assert ((codes & 3) == 2).mean() > 0.99             # block-sum path throughout
    simt = _simt(qa, qb, sa, sb, alpha, 0, 0)
    st = _lib.compare_stats(simt, out)
    assert st["mismatches"] == 0, st
    got = out.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.isfinite(out.float().cpu().numpy()).all()  # no saturation at this data
    a, b, sfa, sfb = (x.cpu().numpy() for x in (qa, qb, sa.view(torch.uint8), sb.view(torch.uint8)))
    band = 11
    ref = _oracle_block(a, b, sfa, sfb, band * BM, BM, 0, S, 0, float(alpha.item()), 0)
    assert nan_equal_mismatches(np.ascontiguousarray(got[band * BM:(band + 1) * BM]), ref, "float16") == 0


def _student_t(shape, g):
    z = torch.randn(shape, generator=g)
    c = sum(torch.randn(shape, generator=g) ** 2 for _ in range(3))
    return z / torch.sqrt(c / 3.0)


@pytest.mark.parametrize("case", [0, 1, 50, 51])
def test_c2_mxfp4_4096_every_output_against_the_oracle(case):
    """C2: cases 0-49 ~N(0,1), 50-99 Student-t(3), bf16 in and out; four of them in full."""
    from emugen_b200.backends.mxfp import build_mxfp_fns

    n = 4096
    g = torch.Generator().manual_seed(1234 + case)
    if case < 50:
        a, b = torch.randn(n, n, generator=g), torch.randn(n, n, generator=g)
    else:
        a, b = _student_t((n, n), g), _student_t((n, n), g)
    quant_fn, _real, emul_fn, _meta = build_mxfp_fns(out_dtype=torch.bfloat16)
    st = quant_fn(a.bfloat16().cuda(), b.bfloat16().cuda())
    out = emul_fn(st)
    assert out.dtype == torch.bfloat16
    got = out.cpu().view(torch.int16).numpy().view(np.uint16)
    ref = oracle.emul_gemm(st.a_fp4.cpu().numpy(), st.b_fp4.cpu().numpy(), st.a_scale.cpu().numpy(),
                           st.b_scale.cpu().numpy(), scale_fmt=1, group_size=32, w_reduce=2,
                           out_mode=oracle.OUT_BF16_VIA_F16)
    assert nan_equal_mismatches(got, ref, "bfloat16") == 0
