"""Drop-in for ``gemm_compare.backends`` (gemm_compare/backends/__init__.py:1-42).

``build_gemm_compare_fns(backend, **kwargs)`` returns ``(quant_fn, real_fn, emul_fn, meta)`` with
unknown keyword arguments filtered per backend, like the reference.  ``quant_fn`` and ``emul_fn``
run on libemugen.so; ``real_fn`` calls the hardware FP4 GEMM from flashinfer (imported lazily).
"""
from __future__ import annotations

from typing import Any, Callable

_MXFP_KW = frozenset({"group_size", "out_dtype", "mm_backend"})
_NVFP_KW = frozenset({"out_dtype", "m_chunk_size", "stage3_rounding", "stage4_rounding"})


def build_gemm_compare_fns(backend: str = "mxfp", **kwargs: Any
                           ) -> tuple[Callable[..., Any], Callable[..., Any], Callable[..., Any], dict[str, Any]]:
    b = backend.lower()
    if b == "mxfp":
        from .mxfp import build_mxfp_fns

        return build_mxfp_fns(**{k: v for k, v in kwargs.items() if k in _MXFP_KW})
    if b == "nvfp":
        from .nvfp import build_nvfp_fns

        return build_nvfp_fns(**{k: v for k, v in kwargs.items() if k in _NVFP_KW})
    raise ValueError(f"unknown backend {backend!r}; expected 'mxfp' or 'nvfp'")


__all__ = ["build_gemm_compare_fns"]
