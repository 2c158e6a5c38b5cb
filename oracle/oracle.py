"""ctypes wrapper around ``_build/liboracle.so`` (the C restatement in ``emul_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` to check results; the product package ``emugen_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

SCALE_E4M3, SCALE_UE8M0 = 0, 1
RZ, RNE = 0, 1
OUT_F16, OUT_BF16_VIA_F16, OUT_F32 = 0, 1, 2

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.is_file():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.oracle_emul_gemm.restype = ctypes.c_int
        L.oracle_emul_gemm.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 7 + [ctypes.c_int] * 5 + [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        L.oracle_emul_gemm_model.restype = ctypes.c_int
        L.oracle_emul_gemm_model.argtypes = L.oracle_emul_gemm.argtypes + [ctypes.c_int] * 4
        L.oracle_swizzle_offset.restype = ctypes.c_int64
        L.oracle_swizzle_offset.argtypes = [ctypes.c_int64] * 3
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def emul_gemm(a_fp4, b_fp4, sfa, sfb, *, scale_fmt, group_size, w_reduce, r3=RZ, r4=RZ,
              alpha=None, out_mode=OUT_F16, nthreads=None, align3=0, align4=0, align_rm=RZ,
              order=0) -> np.ndarray:
    """Oracle emulated GEMM on numpy arrays.  Returns uint16 bits (f16 / bf16) or float32.
    align3 / align4 / align_rm / order select the accumulator model (all 0: the reference's)."""
    a = np.ascontiguousarray(a_fp4, dtype=np.uint8)
    b = np.ascontiguousarray(b_fp4, dtype=np.uint8)
    sa = np.ascontiguousarray(sfa).view(np.uint8)
    sb = np.ascontiguousarray(sfb).view(np.uint8)
    M, N, K = a.shape[0], b.shape[0], a.shape[1] * 2
    assert b.shape[1] * 2 == K
    out = np.empty((M, N), dtype=np.float32 if out_mode == OUT_F32 else np.uint16)
    al = None if alpha is None else np.array([alpha], dtype=np.float32)
    nt = nthreads or os.cpu_count() or 1
    rc = lib().oracle_emul_gemm_model(_ptr(a), _ptr(b), _ptr(sa), _ptr(sb), M, N, K, sa.shape[0], sa.shape[1],
                                      sb.shape[0], sb.shape[1], scale_fmt, group_size, w_reduce, r3, r4,
                                      None if al is None else _ptr(al), out_mode, _ptr(out), nt,
                                      align3, align4, align_rm, order)
    if rc != 0:
        raise ValueError(f"oracle rejected arguments (code {rc})")
    return out


def swizzle_offset(r: int, c: int, cols_pad: int) -> int:
    return int(lib().oracle_swizzle_offset(r, c, cols_pad))
