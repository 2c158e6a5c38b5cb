"""Drop-in for ``gemm_compare.backends.nvfp`` (gemm_compare/backends/nvfp.py:1-221).

Same state dataclass, rollout dict format and builder signatures.  ``quant_fn`` computes the global
scales and alpha on the device (no ``.item()`` round trips) and quantises with libemugen's NVFP4
kernel (the flashinfer fp4_quantize recipe, standing in for the absent ``nvfp.ops.scaled_fp4_quant``);
``emul_fn`` is libemugen's emulated GEMM, bit-exact to the reference C++ emulator.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from .. import _lib
from ..nvfp_cpp_emul import RZ, emulated_scaled_fp4_mm

FLOAT4_E2M1_MAX = 6.0
FLOAT8_E4M3_MAX = 448.0


def global_scale_nvfp(t: torch.Tensor) -> torch.Tensor:
    """f32(2688 / max|t|) as a float32[1] tensor on t's device (reference nvfp.py:24-27)."""
    gs, _, _ = _lib.nvfp4_global_scales(t, t)
    return gs if t.is_cuda else gs.cpu()


@dataclass
class NVFPQuantState:
    a_fp4: torch.Tensor
    b_fp4: torch.Tensor
    scale_a: torch.Tensor
    scale_b: torch.Tensor
    global_scale_a: torch.Tensor
    global_scale_b: torch.Tensor
    alpha: torch.Tensor
    out_dtype: torch.dtype
    w_reduce: int
    group_size: int
    m_chunk_size: int
    stage3_rounding: int
    stage4_rounding: int


def _dtype_to_str(dt: torch.dtype) -> str:
    return str(dt).removeprefix("torch.")


def _dtype_from_str(s: str) -> torch.dtype:
    return getattr(torch, s.removeprefix("torch."))


def nvfp_quant_state_to_cpu_dict(state: NVFPQuantState, *, include_inputs: bool = False) -> dict[str, Any]:
    """Portable dict, same keys as the reference rollout format (nvfp.py:57-75)."""
    return {
        "kind": "nvfp",
        "a_fp4": state.a_fp4.detach().cpu().contiguous(),
        "b_fp4": state.b_fp4.detach().cpu().contiguous(),
        "scale_a": state.scale_a.detach().cpu().contiguous(),
        "scale_b": state.scale_b.detach().cpu().contiguous(),
        "global_scale_a": state.global_scale_a.detach().cpu().contiguous(),
        "global_scale_b": state.global_scale_b.detach().cpu().contiguous(),
        "alpha": state.alpha.detach().cpu().contiguous(),
        "out_dtype": _dtype_to_str(state.out_dtype),
        "w_reduce": int(state.w_reduce),
        "group_size": int(state.group_size),
        "m_chunk_size": int(state.m_chunk_size),
        "stage3_rounding": int(state.stage3_rounding),
        "stage4_rounding": int(state.stage4_rounding),
    }


def nvfp_quant_state_from_dict(d: dict[str, Any], *, device: str | torch.device) -> NVFPQuantState:
    if d.get("kind") != "nvfp":
        raise ValueError(f"expected NVFP state dict, got kind={d.get('kind')!r}")
    return NVFPQuantState(
        a_fp4=d["a_fp4"].to(device), b_fp4=d["b_fp4"].to(device), scale_a=d["scale_a"].to(device),
        scale_b=d["scale_b"].to(device), global_scale_a=d["global_scale_a"].to(device),
        global_scale_b=d["global_scale_b"].to(device), alpha=d["alpha"].to(device),
        out_dtype=_dtype_from_str(d["out_dtype"]), w_reduce=int(d["w_reduce"]), group_size=int(d["group_size"]),
        m_chunk_size=int(d["m_chunk_size"]), stage3_rounding=int(d["stage3_rounding"]),
        stage4_rounding=int(d["stage4_rounding"]))


def build_nvfp_emul_fn(*, out_dtype: torch.dtype = torch.float16, m_chunk_size: int = 128,
                       stage3_rounding: int | None = None, stage4_rounding: int | None = None):
    """Emulation only (reference nvfp.py:98-130).  Like the reference, the result is fp16 whatever
    ``out_dtype`` says: the C++ emulator it replaces always returns fp16."""
    if stage3_rounding is None:
        stage3_rounding = RZ
    if stage4_rounding is None:
        stage4_rounding = RZ

    def emul_fn(state: NVFPQuantState) -> torch.Tensor:
        return emulated_scaled_fp4_mm(state.a_fp4, state.b_fp4, state.scale_a, state.scale_b, state.alpha,
                                      m_chunk_size=state.m_chunk_size, stage3_rounding=state.stage3_rounding,
                                      stage4_rounding=state.stage4_rounding)

    meta: dict[str, Any] = {"backend": "nvfp", "out_dtype": str(out_dtype), "emulation_only": True}
    return emul_fn, meta


def quantize_nvfp4(x: torch.Tensor, global_scale: torch.Tensor):
    """(packed uint8 [M, K/2], swizzled scales as float8_e4m3fn [pad128(M), pad4(K/16)])."""
    q, sf = _lib.quant_nvfp4(x, global_scale)
    return q, sf.view(torch.float8_e4m3fn)


def build_nvfp_fns(*, out_dtype: torch.dtype = torch.float16, m_chunk_size: int = 128,
                   stage3_rounding: int | None = None, stage4_rounding: int | None = None,
                   return_pseudo: bool = False):
    """(quant_fn, real_fn, emul_fn, meta) like the reference (nvfp.py:149-221)."""
    if stage3_rounding is None:
        stage3_rounding = RZ
    if stage4_rounding is None:
        stage4_rounding = RZ
    emul_fn, _ = build_nvfp_emul_fn(out_dtype=out_dtype, m_chunk_size=m_chunk_size,
                                    stage3_rounding=stage3_rounding, stage4_rounding=stage4_rounding)

    def quant_fn(a: torch.Tensor, b: torch.Tensor) -> NVFPQuantState:
        a_gs, b_gs, alpha = _lib.nvfp4_global_scales(a, b)
        a_fp4, scale_a = quantize_nvfp4(a, a_gs)
        b_fp4, scale_b = quantize_nvfp4(b, b_gs)
        return NVFPQuantState(a_fp4=a_fp4, b_fp4=b_fp4, scale_a=scale_a, scale_b=scale_b, global_scale_a=a_gs,
                              global_scale_b=b_gs, alpha=alpha, out_dtype=out_dtype, w_reduce=4, group_size=16,
                              m_chunk_size=m_chunk_size, stage3_rounding=stage3_rounding,
                              stage4_rounding=stage4_rounding)

    def real_fn(state: NVFPQuantState) -> torch.Tensor:
        """Hardware NVFP4 GEMM.  The reference calls the absent ``nvfp.ops.cutlass_scaled_fp4_mm``;
        the installed stand-in is flashinfer.gemm.mm_fp4 with NVFP4 block scales."""
        import flashinfer

        return flashinfer.gemm.mm_fp4(state.a_fp4, state.b_fp4.T, state.scale_a.view(torch.uint8),
                                      state.scale_b.view(torch.uint8).T, state.alpha, state.out_dtype,
                                      block_size=16, use_nvfp4=True)

    meta: dict[str, Any] = {"backend": "nvfp", "out_dtype": str(out_dtype)}
    if return_pseudo:
        from ..pseudo import build_nvfp_pseudo_fn

        pseudo_fn, _ = build_nvfp_pseudo_fn()
        return quant_fn, real_fn, emul_fn, pseudo_fn, meta
    return quant_fn, real_fn, emul_fn, meta
