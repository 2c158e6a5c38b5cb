"""The registered torch operators (emugen_b200.ops) without a GPU: they exist under torch.ops.emugen,
and their fake implementations give the output shape and dtype that torch.compile traces with."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import emugen_b200.ops  # noqa: F401  (registers torch.ops.emugen.*)


def test_ops_are_registered():
    for name in ("gemm", "emulated_scaled_fp4_mm", "emulated_mxfp4_mm"):
        assert hasattr(torch.ops.emugen, name)


def test_fake_shapes_and_dtypes():
    with FakeTensorMode():
        a = torch.empty(7, 64, dtype=torch.uint8)
        b = torch.empty(300, 64, dtype=torch.uint8)
        sa = torch.empty(128, 8, dtype=torch.uint8)
        sb = torch.empty(384, 8, dtype=torch.uint8)
        al = torch.empty(1, dtype=torch.float32)
        out = torch.ops.emugen.emulated_scaled_fp4_mm(a, b, sa.view(torch.float8_e4m3fn), sb.view(torch.float8_e4m3fn), al)
        assert out.shape == (7, 300) and out.dtype == torch.float16
        out = torch.ops.emugen.emulated_mxfp4_mm(a, b, sa[:, :4], sb[:, :4])
        assert out.shape == (7, 300) and out.dtype == torch.float16
        for mode, dt in ((0, torch.float16), (1, torch.bfloat16), (2, torch.float32)):
            out = torch.ops.emugen.gemm(a, b, sa, sb, al, 0, 16, 4, 0, 0, mode)
            assert out.shape == (7, 300) and out.dtype == dt
