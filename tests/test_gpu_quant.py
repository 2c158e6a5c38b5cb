"""GPU tests of the FP4 quantisers: structure (layout, padding, nibble order) against exactly
representable inputs, and bit parity with flashinfer's quantiser (the reference quant_fn's
third-party implementation) when flashinfer can build its kernels on this machine."""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def _exact_input(rng, M, K, gs, dtype):
    """Values whose quantisation is exact: each block holds e2m1 values times 2^e with the max 6."""
    codes = rng.integers(0, 16, (M, K)).astype(np.uint8)
    codes[:, ::gs] = 7  # block max = 6 * 2^e
    vals = np.array(E2M1)[codes & 7] * np.where(codes & 8, -1.0, 1.0)
    e = rng.integers(-3, 4, (M, K // gs)).repeat(gs, axis=1)
    x = vals * np.exp2(e)
    return torch.from_numpy(x).to(dtype), codes, e[:, ::gs]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,K", [(1, 64), (130, 256), (256, 4096)])
def test_mxfp4_quant_exact_values(dtype, M, K):
    from emugen_b200 import quant_mxfp4

    rng = np.random.default_rng(M * K)
    x, codes, e = _exact_input(rng, M, K, 32, dtype)
    q, sf = quant_mxfp4(x.cuda())
    q, sf = q.cpu().numpy(), sf.cpu().numpy()
    exp_codes = codes.copy()
    exp_codes[(codes & 7) == 0] = 0  # -0 quantises to +0 code? keep sign bit as produced below
    lo, hi = q & 0xF, q >> 4
    got = np.empty((M, K), dtype=np.uint8)
    got[:, 0::2], got[:, 1::2] = lo, hi
    nz = (codes & 7) != 0
    assert np.array_equal(got[nz], codes[nz])
    assert np.all((got[~nz] & 7) == 0)
    G = K // 32
    for r in range(0, M, max(1, M // 7)):
        for g in range(G):
            assert sf.reshape(-1)[oracle.swizzle_offset(r, g, sf.shape[1])] == 127 + e[r, g]
    assert sf.shape == ((M + 127) // 128 * 128, (G + 3) // 4 * 4)


def test_quant_padding_is_zero():
    from emugen_b200 import quant_mxfp4, quant_nvfp4

    x = torch.randn(130, 96, dtype=torch.float16, device="cuda")
    _, sf = quant_mxfp4(x)  # 3 scale columns padded to 4, 130 rows padded to 256
    s = sf.cpu().numpy().reshape(-1)
    for r in range(256):
        for c in range(4):
            v = s[oracle.swizzle_offset(r, c, 4)]
            if r >= 130 or c >= 3:
                assert v == 0
    gs = torch.tensor([1.0], device="cuda")
    _, sf = quant_nvfp4(torch.randn(5, 80, dtype=torch.bfloat16, device="cuda"), gs)
    s = sf.cpu().numpy().reshape(-1)
    assert all(s[oracle.swizzle_offset(r, c, 8)] == 0 for r in range(128) for c in range(8) if r >= 5 or c >= 5)


def _flashinfer_fp4_quantize():
    try:
        import flashinfer
        from flashinfer import fp4_quantize
        fp4_quantize(torch.randn(128, 64, dtype=torch.float16, device="cuda"), torch.tensor([1.0], device="cuda"),
                     16, False, True)
        return flashinfer
    except Exception as e:  # flashinfer missing or its JIT build unavailable
        pytest.skip(f"flashinfer fp4_quantize unavailable: {type(e).__name__}: {e}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,K", [(128, 256), (257, 1024), (1, 4096)])
def test_quant_bit_parity_with_flashinfer(dtype, M, K):
    fi = _flashinfer_fp4_quantize()
    from emugen_b200 import nvfp4_global_scales, quant_mxfp4, quant_nvfp4

    g = torch.Generator().manual_seed(M + K)
    x = (torch.randn(M, K, generator=g) * torch.exp(torch.randn(M, 1, generator=g))).to(dtype).cuda()
    x[0, :7] = 0
    gs, _, _ = nvfp4_global_scales(x, x)
    q_ref, sf_ref = fi.fp4_quantize(x, gs, 16, False, True)
    q, sf = quant_nvfp4(x, gs)
    assert torch.equal(q.cpu(), q_ref.view(torch.uint8).cpu())
    assert torch.equal(sf.cpu().reshape(-1), sf_ref.view(torch.uint8).cpu().reshape(-1))
    q_ref, sf_ref = fi.mxfp4_quantize(x)
    q, sf = quant_mxfp4(x)
    assert torch.equal(q.cpu(), q_ref.view(torch.uint8).cpu())
    assert torch.equal(sf.cpu().reshape(-1), sf_ref.view(torch.uint8).cpu().reshape(-1))


def test_global_scales_match_reference_recipe():
    from emugen_b200 import nvfp4_global_scales

    a = torch.randn(300, 500, dtype=torch.float16) * 3
    b = torch.randn(200, 500, dtype=torch.float16)
    gsa, gsb, alpha = nvfp4_global_scales(a.cuda(), b.cuda())
    # reference gemm_compare/backends/nvfp.py:24-27, 176 in Python doubles
    amax_a = torch.abs(a).max().to(torch.float32).item()
    amax_b = torch.abs(b).max().to(torch.float32).item()
    ga = np.float32(448.0 * 6.0 / (amax_a if amax_a > 0 else 1.0))
    gb = np.float32(448.0 * 6.0 / (amax_b if amax_b > 0 else 1.0))
    al = np.float32(1.0 / max(float(ga) * float(gb), 1e-8))
    assert gsa.item() == float(ga) and gsb.item() == float(gb) and alpha.item() == float(al)
    z = torch.zeros(4, 16, dtype=torch.bfloat16, device="cuda")
    gz, _, _ = nvfp4_global_scales(z, z)
    assert gz.item() == 2688.0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_global_scales_vector_and_tail_paths(dtype):
    """The amax reads 16-byte vectors where the pointer allows and single elements elsewhere: a numel
    that is not a multiple of 8, a pointer one element past a 16-byte boundary, the maximum in the
    tail, an infinity and a NaN all give the reference's scale (gemm_compare/backends/nvfp.py:24-27)."""
    from emugen_b200 import nvfp4_global_scales

    def want(x):
        am = torch.abs(x.float()).max().item()
        return np.float32(448.0 * 6.0 / (am if am > 0 else 1.0))

    base = torch.randn(4099, dtype=torch.float32).to(dtype).cuda()
    for x in (base[:4097], base[1:4098]):
        y = x.clone() if x.data_ptr() % 16 == 0 else x
        y[-1] = 9.0
        g, _, _ = nvfp4_global_scales(y, y)
        w = want(y.cpu())
        assert g.item() == float(w), (dtype, y.data_ptr() % 16)
    z = base[:4096].clone()
    z[77] = -float("inf")
    g, _, _ = nvfp4_global_scales(z, z)
    assert g.item() == float(want(z.cpu())) == 0.0          # 2688 / inf
    z[100] = float("nan")
    g, _, _ = nvfp4_global_scales(z, z)
    assert g.item() == float(want(z.cpu())) == 2688.0       # NaN > 0 is false: the reference falls back to 1.0


def _parity(fi, x, gs):
    from emugen_b200 import quant_mxfp4, quant_nvfp4

    q_ref, sf_ref = fi.fp4_quantize(x, gs, 16, False, True)
    q, sf = quant_nvfp4(x, gs)
    nv = (int((q.cpu() != q_ref.view(torch.uint8).cpu()).sum()),
          int((sf.cpu().reshape(-1) != sf_ref.view(torch.uint8).cpu().reshape(-1)).sum()))
    q_ref, sf_ref = fi.mxfp4_quantize(x)
    q, sf = quant_mxfp4(x)
    mx = (int((q.cpu() != q_ref.view(torch.uint8).cpu()).sum()),
          int((sf.cpu().reshape(-1) != sf_ref.view(torch.uint8).cpu().reshape(-1)).sum()))
    return nv, mx


@pytest.mark.parametrize("recipe", ["benchmark_outlier_columns_fp16", "student_t3_bf16"])
def test_quant_bit_parity_on_benchmark_data(recipe):
    """The benchmark's data recipes: |N(0,1)| fp16 with 1% of K columns x100 (NVFP4 8192^3 case; 1024
    rows of it), and Student-t(3) bf16 (the MXFP4 suite's second half)."""
    fi = _flashinfer_fp4_quantize()
    from emugen_b200 import nvfp4_global_scales

    g = torch.Generator().manual_seed(7)
    if recipe.startswith("benchmark"):
        x = torch.randn(1024, 8192, generator=g).abs_()
        x[:, torch.randperm(8192, generator=g)[:82]] *= 100.0
        x = x.half()
    else:
        z = torch.randn(1024, 4096, generator=g)
        c = sum(torch.randn(1024, 4096, generator=g) ** 2 for _ in range(3))
        x = (z / torch.sqrt(c / 3.0)).bfloat16()
    x = x.cuda()
    gs, _, _ = nvfp4_global_scales(x, x)
    assert _parity(fi, x, gs) == ((0, 0), (0, 0))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quant_bit_parity_on_special_values(dtype):
    """All-zero blocks, subnormal inputs, +-inf and NaN inside otherwise normal blocks, quantised with a
    fixed global scale (the global scale of such operands has its own test above)."""
    fi = _flashinfer_fp4_quantize()

    g = torch.Generator().manual_seed(11)
    x = torch.randn(256, 1024, generator=g)
    x[0:8, :] = 0.0                                    # whole rows of zero blocks
    x[8:16, 0:64] = 0.0                                # zero blocks inside a row
    tiny = torch.finfo(dtype).tiny
    x[16:32, :] = torch.randn(16, 1024, generator=g) * tiny * 0.25   # subnormal inputs
    x[32, 5] = float("inf")
    x[33, 100] = float("-inf")
    x[34, 300] = float("nan")
    x[35, 17:19] = float("nan")
    x = x.to(dtype).cuda()
    gs = torch.tensor([448.0 * 6.0 / 4.0], device="cuda")
    nv, mx = _parity(fi, x, gs)
    assert nv == (0, 0) and mx == (0, 0), (nv, mx)
