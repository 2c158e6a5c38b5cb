"""Drop-in for the reference package ``mxfp_cpp_emul`` (mxfp_cpp_emul/mxfp_cpp_emul/__init__.py).

``emulated_mxfp4_mm`` matches the reference pybind export (mxfp_cpp_emul/mxfp_cpp_emul/csrc/
mxfp_emulation.cpp:98-106, 168-181): same arguments, same TORCH_CHECK messages, same fp16 result
bit for bit, computed by libemugen.so on the GPU.  Scales are uint8 UE8M0 bytes (as returned by
flashinfer.mxfp4_quantize).  ``configure_jit`` / ``JIT_EXTRA_*`` are kept for import
compatibility only; CPU tensors are computed on the current CUDA device and copied back.
"""
from __future__ import annotations

from typing import Any

import torch

from . import _lib

JIT_EXTRA_CFLAGS: list[str] = []
JIT_EXTRA_LDFLAGS: list[str] = []
JIT_EXTRA_INCLUDE_PATHS: list[str] = []

RZ = 0
RNE = 1


def configure_jit(*, extra_cflags: list[str] | None = None, extra_ldflags: list[str] | None = None,
                  extra_include_paths: list[str] | None = None, **kwargs: Any) -> None:
    """Accepted for compatibility with the reference loader; the library is not JIT-built."""
    if extra_cflags is not None:
        JIT_EXTRA_CFLAGS[:] = extra_cflags
    if extra_ldflags is not None:
        JIT_EXTRA_LDFLAGS[:] = extra_ldflags
    if extra_include_paths is not None:
        JIT_EXTRA_INCLUDE_PATHS[:] = extra_include_paths


def emulated_mxfp4_mm(a_fp4: torch.Tensor, b_fp4: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                      group_size: int = 32, m_chunk_size: int = 128, stage3_rounding: int = 0,
                      stage4_rounding: int = 0) -> torch.Tensor:
    """MXFP4 scaled GEMM emulation -> [M, N] float16 (reference mxfp_emulation.cpp:98-166)."""
    if a_fp4.dim() != 2 or b_fp4.dim() != 2:
        raise RuntimeError("a_fp4, b_fp4 must be 2D")
    if int(group_size) != 32:
        raise RuntimeError("only MXFP4 group_size=32 is supported")
    if int(m_chunk_size) <= 0:
        raise RuntimeError("m_chunk_size must be positive")
    for name, s in (("scale_a", scale_a), ("scale_b", scale_b)):
        if s.dtype != torch.uint8:
            raise TypeError(f"{name} must be uint8 UE8M0 bytes, got {s.dtype}")
    return _lib.gemm(a_fp4, b_fp4, scale_a, scale_b, fmt=_lib.EMU_FMT_MXFP4, group_size=32, w_reduce=2,
                     stage3_rounding=_lib.EMU_RZ if int(stage3_rounding) == 0 else _lib.EMU_RNE,
                     stage4_rounding=_lib.EMU_RZ if int(stage4_rounding) == 0 else _lib.EMU_RNE,
                     alpha=None, out_mode=_lib.EMU_OUT_F16)


__all__ = ["RZ", "RNE", "JIT_EXTRA_CFLAGS", "JIT_EXTRA_LDFLAGS", "JIT_EXTRA_INCLUDE_PATHS", "configure_jit",
           "emulated_mxfp4_mm"]
