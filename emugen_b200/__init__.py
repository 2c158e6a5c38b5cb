"""emugen_b200 — EmuGen's emulated NVFP4 / MXFP4 scaled GEMM on NVIDIA B200 (sm_100a).

The compute lives in ``libemugen.so`` (C ABI in include/emugen.h, CUDA kernels in csrc/).  The
Python modules mirror the reference interfaces that call it:

  emugen_b200.nvfp_cpp_emul   <- nvfp_cpp_emul            (emulated_scaled_fp4_mm, RZ, RNE)
  emugen_b200.mxfp_cpp_emul   <- mxfp_cpp_emul            (emulated_mxfp4_mm)
  emugen_b200.emulation       <- search.emulation         (MMAEngine, emulate_nvfp_scaled_fp4_mm, ...)
  emugen_b200.backends        <- gemm_compare.backends    (build_nvfp_fns, build_mxfp_fns, states)
"""
from . import _lib
from ._lib import EmuError, gemm, nvfp4_global_scales, quant_mxfp4, quant_nvfp4

__all__ = ["EmuError", "gemm", "nvfp4_global_scales", "quant_mxfp4", "quant_nvfp4", "load_library"]


def load_library():
    """Load libemugen.so (raises if it has not been built)."""
    return _lib.load()
