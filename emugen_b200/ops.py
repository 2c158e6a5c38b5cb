"""The emulated GEMMs as registered torch operators: ``torch.ops.emugen.*``.

Registered with ``torch.library.custom_op`` together with a fake (shape-only) implementation, so that
``torch.compile`` traces through them as single opaque nodes with known [M, N] outputs, and CUDA-graph
capture records their launches (the library allocates only through torch's allocator and does not
synchronise the host).  Each op calls the same C ABI as the Python drop-ins:

  torch.ops.emugen.emulated_scaled_fp4_mm  <- nvfp_cpp_emul.emulated_scaled_fp4_mm (nvfp_emulation.cpp:90-156)
  torch.ops.emugen.emulated_mxfp4_mm       <- mxfp_cpp_emul.emulated_mxfp4_mm     (mxfp_emulation.cpp:98-166)
  torch.ops.emugen.gemm                     every format / block size / rounding / output mode (emu_gemm_ws)

Importing this module registers the ops (``import emugen_b200.ops``); the reference has no torch-op
registration of its own (it loads its C++ emulators as Python extension modules).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_OUT_DTYPE = {_lib.EMU_OUT_F16: torch.float16, _lib.EMU_OUT_BF16_VIA_F16: torch.bfloat16,
              _lib.EMU_OUT_F32: torch.float32}


def _rounding(code: int) -> int:
    """The C++ emulators' rounding codes: 0 is RZ, any other value RNE."""
    return _lib.EMU_RZ if int(code) == 0 else _lib.EMU_RNE


@torch.library.custom_op("emugen::gemm", mutates_args=())
def gemm(a_fp4: torch.Tensor, b_fp4: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
         alpha: Optional[torch.Tensor], fmt: int, group_size: int, w_reduce: int, stage3_rounding: int,
         stage4_rounding: int, out_mode: int) -> torch.Tensor:
    """Emulated scaled FP4 GEMM [M, K/2] x [N, K/2] -> [M, N] (fp16 / bf16 / f32 by out_mode)."""
    return _lib.gemm(a_fp4, b_fp4, scale_a, scale_b, fmt=fmt, group_size=group_size, w_reduce=w_reduce,
                     stage3_rounding=stage3_rounding, stage4_rounding=stage4_rounding, alpha=alpha,
                     out_mode=out_mode)


@gemm.register_fake
def _gemm_fake(a_fp4, b_fp4, scale_a, scale_b, alpha, fmt, group_size, w_reduce, stage3_rounding,
               stage4_rounding, out_mode):
    torch._check(a_fp4.dim() == 2 and b_fp4.dim() == 2, lambda: "a_fp4, b_fp4 must be 2D")
    torch._check(a_fp4.shape[1] == b_fp4.shape[1], lambda: "K mismatch between a and b")
    return a_fp4.new_empty((a_fp4.shape[0], b_fp4.shape[0]), dtype=_OUT_DTYPE[out_mode])


@torch.library.custom_op("emugen::emulated_scaled_fp4_mm", mutates_args=())
def emulated_scaled_fp4_mm(a_fp4: torch.Tensor, b_fp4: torch.Tensor, scale_a: torch.Tensor,
                           scale_b: torch.Tensor, alpha: torch.Tensor, m_chunk_size: int = 128,
                           stage3_rounding: int = 0, stage4_rounding: int = 0) -> torch.Tensor:
    """NVFP4 (16-element groups, E4M3 scales, 4 groups per block) -> [M, N] fp16, as the reference's."""
    if int(m_chunk_size) <= 0:
        raise RuntimeError("m_chunk_size must be positive")
    return _lib.gemm(a_fp4, b_fp4, scale_a, scale_b, fmt=_lib.EMU_FMT_NVFP4, group_size=16, w_reduce=4,
                     stage3_rounding=_rounding(stage3_rounding), stage4_rounding=_rounding(stage4_rounding),
                     alpha=alpha, out_mode=_lib.EMU_OUT_F16)


@emulated_scaled_fp4_mm.register_fake
def _nvfp_fake(a_fp4, b_fp4, scale_a, scale_b, alpha, m_chunk_size=128, stage3_rounding=0, stage4_rounding=0):
    torch._check(a_fp4.shape[1] == b_fp4.shape[1], lambda: "K mismatch between a and b")
    return a_fp4.new_empty((a_fp4.shape[0], b_fp4.shape[0]), dtype=torch.float16)


@torch.library.custom_op("emugen::emulated_mxfp4_mm", mutates_args=())
def emulated_mxfp4_mm(a_fp4: torch.Tensor, b_fp4: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                      group_size: int = 32, m_chunk_size: int = 128, stage3_rounding: int = 0,
                      stage4_rounding: int = 0) -> torch.Tensor:
    """MXFP4 (32-element groups, UE8M0 scales, 2 groups per block) -> [M, N] fp16, as the reference's."""
    if int(group_size) != 32:
        raise RuntimeError("only MXFP4 group_size=32 is supported")
    if int(m_chunk_size) <= 0:
        raise RuntimeError("m_chunk_size must be positive")
    return _lib.gemm(a_fp4, b_fp4, scale_a, scale_b, fmt=_lib.EMU_FMT_MXFP4, group_size=32, w_reduce=2,
                     stage3_rounding=_rounding(stage3_rounding), stage4_rounding=_rounding(stage4_rounding),
                     alpha=None, out_mode=_lib.EMU_OUT_F16)


@emulated_mxfp4_mm.register_fake
def _mxfp_fake(a_fp4, b_fp4, scale_a, scale_b, group_size=32, m_chunk_size=128, stage3_rounding=0,
               stage4_rounding=0):
    torch._check(a_fp4.shape[1] == b_fp4.shape[1], lambda: "K mismatch between a and b")
    return a_fp4.new_empty((a_fp4.shape[0], b_fp4.shape[0]), dtype=torch.float16)


__all__ = ["gemm", "emulated_scaled_fp4_mm", "emulated_mxfp4_mm"]
