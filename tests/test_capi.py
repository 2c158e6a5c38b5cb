"""The C-ABI library loads, exports every symbol include/emugen.h declares, and rejects bad
arguments with the reference's messages -- all before any CUDA call, so this runs without a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from emugen_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "emugen.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"EMU_API\s+[\w\s\*]+?\b(emu_\w+)\s*\(", text)))


def test_header_declares_what_binding_expects():
    assert set(declared_symbols()) == set(_lib.SYMBOLS)


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert L.emu_abi_version() == _lib.ABI_VERSION


def _gemm_status(M=4, N=4, K=64, sa=(128, 4), sb=(128, 4), **p):
    L = _lib.load()
    params = _lib.EmuGemmParams(p.get("format", 0), p.get("group_size", 16), p.get("w_reduce", 4),
                                p.get("r3", 0), p.get("r4", 0), p.get("out_mode", 0))
    fake = ctypes.c_void_p(16)  # never dereferenced: validation fails before any device access
    st = L.emu_gemm(fake, fake, fake, fake, M, N, K, sa[0], sa[1], sb[0], sb[1], None, ctypes.byref(params),
                    fake, None)
    return st, L.emu_last_error().decode()


@pytest.mark.parametrize("kw,status,msg", [
    (dict(K=40), 3, "K must be multiple of 16"),
    (dict(K=48), 4, "G = K/16 must be multiple of 4"),
    (dict(format=1, group_size=16, w_reduce=2), 5, "only MXFP4 group_size=32 is supported"),
    (dict(format=1, group_size=32, w_reduce=2, K=96), 4,
     "MXFP emulation (w_reduce=2) requires K/(2*group_size) to be integral (e.g. K divisible by 64)"),
    (dict(format=1, group_size=32, w_reduce=2, K=48), 3, "K must be divisible by group_size"),
    (dict(sa=(100, 4)), 6, "swizzled scale shape must be divisible by 128 and 4"),
    (dict(sb=(128, 6)), 6, "swizzled scale shape must be divisible by 128 and 4"),
    (dict(M=200), 7, "scale rows"),
    (dict(K=256), 7, "scale columns"),
    (dict(w_reduce=3, K=80), 4, "must be divisible by w_reduce"),
    (dict(w_reduce=0), 8, "w_reduce must be in [1, 64]"),
    (dict(r3=2), 1, "rounding must be"),
    (dict(out_mode=7), 1, "unknown out_mode"),
    (dict(format=5), 1, "unknown format"),
])
def test_gemm_validation_messages(kw, status, msg):
    st, err = _gemm_status(**kw)
    assert st == status
    assert msg in err


def test_empty_output_is_ok_without_device():
    st, err = _gemm_status(M=0)
    assert st == 0 and err == ""


def test_quant_validation():
    L = _lib.load()
    fake = ctypes.c_void_p(16)
    assert L.emu_quant_nvfp4(fake, 0, 4, 40, fake, fake, fake, None) == 3
    assert "multiple of 16" in L.emu_last_error().decode()
    assert L.emu_quant_mxfp4(fake, 0, 4, 48, fake, fake, None) == 3
    assert L.emu_quant_mxfp4(fake, 7, 4, 64, fake, fake, None) == 1
    assert L.emu_quant_nvfp4(fake, 0, 4, 64, None, fake, fake, None) == 1


def test_wait_limit_and_status_names():
    """The pipeline-wait bound is a process-wide setting that returns the previous value (no device
    call); EMU_ERR_TIMEOUT has a name."""
    L = _lib.load()
    default = 1 << 31
    prev = L.emu_set_wait_limit(1000)
    try:
        assert prev == default
        assert L.emu_set_wait_limit(-5) == 1000
        assert L.emu_set_wait_limit(0) == default
    finally:
        L.emu_set_wait_limit(prev)
    assert L.emu_status_string(_lib.EMU_ERR_TIMEOUT) == b"EMU_ERR_TIMEOUT"
    assert L.emu_test_hold_first_ready(0) == _lib.EMU_OK


def _batch_status(sets, n=None, out=True, ref=False, stats=True, M=4, N=4, K=64):
    L = _lib.load()
    arr = (_lib.EmuGemmParams * max(len(sets), 1))(*[_lib.EmuGemmParams(*s) for s in sets]) if sets else None
    fake = ctypes.c_void_p(256)  # never dereferenced: validation fails before any device access
    st = L.emu_gemm_batch(fake, fake, fake, fake, M, N, K, 128, 4, 128, 4, None, arr,
                          len(sets) if n is None else n, fake if ref else None, fake if out else None,
                          fake if stats else None, None, 0, None)
    return st, L.emu_last_error().decode()


NV = (0, 16, 4, 0, 0, 0)


@pytest.mark.parametrize("kw,msg", [
    (dict(sets=[]), "params must not be NULL"),
    (dict(sets=[NV], n=0), "n_params must be in [1, 4096]"),
    (dict(sets=[NV], n=5000), "n_params must be in [1, 4096]"),
    (dict(sets=[NV], out=False), "out and ref are both NULL"),
    (dict(sets=[NV], ref=True, stats=False), "stats must not be NULL"),
    (dict(sets=[NV, (1, 32, 2, 0, 0, 0)]), "params[1]: every set must have params[0]'s format"),
    (dict(sets=[NV, (0, 16, 4, 0, 0, 2)]), "params[1]: every set must have params[0]'s format"),
])
def test_gemm_batch_validation(kw, msg):
    st, err = _batch_status(**kw)
    assert st == 1 and msg in err


def test_gemm_batch_checks_every_set_like_emu_gemm():
    st, err = _batch_status([NV, (0, 16, 0, 0, 0, 0)])
    assert st == 8 and "w_reduce must be in [1, 64]" in err
