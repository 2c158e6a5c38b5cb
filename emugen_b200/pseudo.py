"""pseudo_fn: dequantise both FP4 operands on the device and multiply them with a plain GEMM.

Mirrors gemm_compare/backends/nvfp.py:133-146 ``build_nvfp_pseudo_fn`` and mxfp.py:155-165
``build_mxfp_pseudo_fn``.  Dequantisation is libemugen's emu_dequant_fp4; the product is a torch
matmul (cuBLAS), as the reference's ``a @ b.T``.  The reference's MXFP4 version dequantises on the
host with flashinfer and multiplies in f32 on the CPU; here both run on the operands' device.
"""
from __future__ import annotations

from typing import Any

import torch

from . import _lib


def build_nvfp_pseudo_fn():
    def pseudo_fn(state) -> torch.Tensor:
        a = _lib.dequant_fp4(state.a_fp4, state.scale_a, fmt=_lib.EMU_FMT_NVFP4,
                             global_scale=state.global_scale_a).to(state.out_dtype)
        b = _lib.dequant_fp4(state.b_fp4, state.scale_b, fmt=_lib.EMU_FMT_NVFP4,
                             global_scale=state.global_scale_b).to(state.out_dtype)
        return a @ b.T

    meta: dict[str, Any] = {"backend": "nvfp", "pseudo_only": True}
    return pseudo_fn, meta


def build_mxfp_pseudo_fn():
    def pseudo_fn(state) -> torch.Tensor:
        a = _lib.dequant_fp4(state.a_fp4, state.a_scale, fmt=_lib.EMU_FMT_MXFP4)
        b = _lib.dequant_fp4(state.b_fp4, state.b_scale, fmt=_lib.EMU_FMT_MXFP4)
        return a @ b.T

    meta: dict[str, Any] = {"backend": "mxfp", "pseudo_only": True}
    return pseudo_fn, meta
