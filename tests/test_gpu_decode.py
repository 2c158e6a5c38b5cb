"""GPU parity of the decode-shape kernels of gemm_decode.cu -- the decode kernel (2 <= M < 128 rows of A,
N >= 8192 columns, stage 1 on the integer MMA) and the one-row kernel (M = 1, N >= 32768) -- bit for bit:
sampled columns (the first, the ragged last tile, a random set) against the C oracle, and every output
against the skinny kernels on the same data -- the scales of B passed at an odd address, which both
kernels decline (they read them a word at a time) and the skinny kernels read byte by byte."""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden.make_golden import gen_inputs, pad, swizzle
from tests.golden_cases import nan_equal_mismatches

CASES = [
    # kind, data, M, N, K, w_reduce, r3, r4, out_mode
    ("nvfp", "normal", 8, 8192, 4096, 4, 0, 0, 0),           # the reference's block size (fixed at compile time)
    ("nvfp", "outliers", 2, 8200, 1088, 4, 1, 0, 1),         # ragged last tile; a window and a half chunk
    ("nvfp", "raw_nan_scales", 5, 8192, 2048, 4, 0, 1, 0),   # NaN scale codes in A and B
    ("nvfp", "fp16_round", 16, 8192, 512, 4, 1, 1, 2),       # stage-1 rounding (flagged groups)
    ("nvfp", "cancel", 9, 8256, 1024, 1, 0, 0, 2),           # block size read at run time
    ("nvfp", "huge_scales", 33, 8192, 640, 8, 0, 0, 0),      # three 16-row passes
    # blocks of 64 / 32 groups of the largest E4M3 scales: the int64 block sums take the int64 -> f64
    # conversion (exact below 2^53, i.e. up to 64 groups), not the 1.5 * 2^52 bias of blocks up to 16
    ("nvfp", "huge_scales", 8, 8192, 2048, 64, 1, 0, 2),
    ("nvfp", "tiny_scales", 127, 8192, 256, 16, 1, 0, 2),    # one block: R3
    ("nvfp", "abs_normal", 24, 9000, 64, 4, 0, 1, 0),        # K = one block
    ("mxfp", "normal", 8, 8192, 4096, 2, 0, 0, 1),
    ("mxfp", "student_t", 3, 8200, 1088, 2, 1, 0, 2),
    ("mxfp", "raw_scales_full", 16, 8192, 512, 2, 0, 1, 2),  # UE8M0 0 and 255 (inf)
    ("mxfp", "subnormal_acc", 17, 8192, 1024, 1, 1, 1, 0),
    ("mxfp", "flt_max", 7, 8192, 128, 2, 0, 0, 2),
    ("mxfp", "fp16_round", 12, 8320, 2112, 3, 0, 0, 1),     # w_reduce 3 (run time), 66 groups
    # one row of A (emul_gemm_gemv_kernel): 4096-element windows, several and partial, ragged column tiles
    ("nvfp", "normal", 1, 32808, 1024, 4, 0, 0, 0),
    ("nvfp", "raw_nan_scales", 1, 32768, 9216, 4, 1, 1, 1),  # three windows; NaN scale codes in A and B
    ("nvfp", "fp16_round", 1, 32768, 4160, 1, 0, 1, 2),      # flagged groups; a 64-element last window
    ("nvfp", "huge_scales", 1, 33000, 5120, 16, 1, 0, 0),    # block size 16 (run time)
    ("nvfp", "huge_scales", 1, 32768, 4096, 32, 0, 1, 2),    # block size 32: int64 -> f64 conversion
    ("mxfp", "raw_scales_full", 1, 32768, 8256, 2, 0, 1, 2), # UE8M0 0 and 255 (inf)
    ("mxfp", "subnormal_acc", 1, 32900, 2048, 1, 1, 1, 0),
    ("mxfp", "normal", 1, 32768, 1024, 2, 0, 0, 1),
]
IDS = [f"{c[0]}-{c[1]}-{c[2]}x{c[3]}x{c[4]}-wr{c[5]}" for c in CASES]


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _unswizzle(swz, rows, cols):
    """Swizzled 128x4 scale buffer -> linear [rows, cols] bytes (inverse of make_golden.swizzle)."""
    rp, cp = swz.shape
    t = swz.reshape(rp // 128, cp // 4, 32, 4, 4).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(t.reshape(rp, cp))[:rows, :cols]


def _case(kind, data, M, N, K):
    rng = np.random.default_rng(zlib.crc32(f"decode-{kind}-{data}-{M}-{N}-{K}".encode()))
    a, b, sfa, sfb, alpha = gen_inputs(dict(kind=kind, data=data, M=M, N=N, K=K), rng)
    return rng, a, b, sfa, sfb, alpha


def _nan_mask(x, out):
    if out == 2:
        return np.isnan(x)
    if out == 1:   # bf16 bits
        return ((x & 0x7F80) == 0x7F80) & ((x & 0x7F) != 0)
    return ((x & 0x7C00) == 0x7C00) & ((x & 0x3FF) != 0)   # fp16 bits


def _same(x, y, out):
    """Bit equality of two outputs of the same dtype, any NaN equal to any NaN."""
    xn, yn = _nan_mask(x, out), _nan_mask(y, out)
    if out == 2:
        x, y = x.view(np.uint32), y.view(np.uint32)
    return np.array_equal(xn, yn) and np.array_equal(x[~xn], y[~yn])


def _equal(got, ref, out):
    if out == 2:
        gn, rn = np.isnan(got), np.isnan(ref)
        return np.array_equal(gn, rn) and np.array_equal(got[~gn].view(np.uint32), ref[~rn].view(np.uint32))
    return nan_equal_mismatches(got, ref, "bfloat16" if out == 1 else "float16") == 0


@pytest.mark.gpu
@pytest.mark.parametrize("kind,data,M,N,K,wr,r3,r4,out", CASES, ids=IDS)
def test_decode_vs_oracle_and_skinny(kind, data, M, N, K, wr, r3, r4, out):
    from emugen_b200 import _lib

    rng, a, b, sfa, sfb, alpha = _case(kind, data, M, N, K)
    gs = 16 if kind == "nvfp" else 32
    fmt = 0 if kind == "nvfp" else 1
    al = float(alpha) if kind == "nvfp" else None
    ta, tb, tsa, tsb = (torch.from_numpy(x).cuda() for x in (a, b, sfa, sfb))
    kw = dict(fmt=fmt, group_size=gs, w_reduce=wr, stage3_rounding=r3, stage4_rounding=r4,
              alpha=None if al is None else torch.tensor([al], device="cuda"), out_mode=out)
    assert tsb.data_ptr() % 4 == 0
    got = _lib.gemm(ta, tb, tsa, tsb, path="simt", **kw)       # M < 128, no workspace: the decode / one-row kernel

    # the same scales at an odd address: the skinny kernel
    buf = torch.zeros(tsb.numel() + 1, dtype=torch.uint8, device="cuda")
    odd = buf[1:].view(tsb.shape)
    odd.copy_(tsb)
    skinny = _lib.gemm(ta, tb, tsa, odd, path="simt", **kw)
    g = got.cpu().numpy() if out == 2 else _bits(got)
    s = skinny.cpu().numpy() if out == 2 else _bits(skinny)
    assert _same(g, s, out)

    cols = np.unique(np.concatenate([np.arange(8), np.arange(N - min(N, 136), N),
                                     rng.choice(N, 96, replace=False)]))
    G = K // gs
    sb_lin = _unswizzle(sfb, N, G)
    ref = oracle.emul_gemm(a, b[cols], sfa, swizzle(sb_lin[cols], pad(len(cols), 128), pad(G, 4)),
                           scale_fmt=fmt, group_size=gs, w_reduce=wr, r3=r3, r4=r4, alpha=al, out_mode=out)
    assert _equal(g[:, cols], ref, out)


def test_unswizzle_inverts_swizzle():
    rng = np.random.default_rng(3)
    lin = rng.integers(0, 256, (300, 37), dtype=np.uint8)
    swz = swizzle(lin, pad(300, 128), pad(37, 4))
    assert np.array_equal(_unswizzle(swz, 300, 37), lin)
