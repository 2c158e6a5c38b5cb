"""The registered operators (torch.ops.emugen.*) on the GPU: bit-equal to the drop-in modules, traced by
torch.compile (fullgraph) as single nodes, and recorded by CUDA-graph capture with replays bit-equal to
the eager call -- on the CUDA-core path and on the tensor-core path."""
import pytest
import torch

import emugen_b200.ops  # noqa: F401

pytestmark = pytest.mark.gpu


def _nvfp_case(S, seed):
    from emugen_b200 import nvfp4_global_scales, quant_nvfp4

    g = torch.Generator().manual_seed(seed)
    a = torch.randn(S, S, generator=g).half().cuda()
    b = torch.randn(S, S, generator=g).half().cuda()
    gsa, gsb, alpha = nvfp4_global_scales(a, b)
    (qa, sa), (qb, sb) = quant_nvfp4(a, gsa), quant_nvfp4(b, gsb)
    return qa, qb, sa.view(torch.float8_e4m3fn), sb.view(torch.float8_e4m3fn), alpha


def _mxfp_case(S, seed):
    from emugen_b200 import quant_mxfp4

    g = torch.Generator().manual_seed(seed)
    a = torch.randn(S, S, generator=g).bfloat16().cuda()
    b = torch.randn(S, S, generator=g).bfloat16().cuda()
    (qa, sa), (qb, sb) = quant_mxfp4(a), quant_mxfp4(b)
    return qa, qb, sa, sb


def _same(x, y):
    return torch.equal(x.view(torch.int16), y.view(torch.int16))


@pytest.mark.parametrize("S", [256, 1024])   # 256: CUDA-core kernel; 1024: tensor-core kernel
def test_ops_equal_drop_ins(S):
    from emugen_b200 import mxfp_cpp_emul, nvfp_cpp_emul

    qa, qb, sa, sb, alpha = _nvfp_case(S, 1)
    ref = nvfp_cpp_emul.emulated_scaled_fp4_mm(qa, qb, sa, sb, alpha)
    assert _same(torch.ops.emugen.emulated_scaled_fp4_mm(qa, qb, sa, sb, alpha), ref)
    assert _same(torch.ops.emugen.gemm(qa, qb, sa.view(torch.uint8), sb.view(torch.uint8), alpha, 0, 16, 4, 0, 0, 0), ref)
    qa, qb, sa, sb = _mxfp_case(S, 2)
    ref = mxfp_cpp_emul.emulated_mxfp4_mm(qa, qb, sa, sb)
    assert _same(torch.ops.emugen.emulated_mxfp4_mm(qa, qb, sa, sb), ref)


def test_torch_compile_traces_the_op():
    qa, qb, sa, sb, alpha = _nvfp_case(256, 3)

    def f(qa, qb, sa, sb, alpha):
        return torch.ops.emugen.emulated_scaled_fp4_mm(qa, qb, sa, sb, alpha).float() * 2.0

    cf = torch.compile(f, backend="aot_eager", fullgraph=True)
    assert torch.equal(cf(qa, qb, sa, sb, alpha), f(qa, qb, sa, sb, alpha))


@pytest.mark.parametrize("S", [256, 1024])
def test_cuda_graph_capture_and_replay(S):
    qa, qb, sa, sb, alpha = _nvfp_case(S, 4)
    eager = torch.ops.emugen.emulated_scaled_fp4_mm(qa, qb, sa, sb, alpha)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            torch.ops.emugen.emulated_scaled_fp4_mm(qa, qb, sa, sb, alpha)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = torch.ops.emugen.emulated_scaled_fp4_mm(qa, qb, sa, sb, alpha)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert _same(out, eager)
    del g
