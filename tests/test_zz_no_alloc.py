"""emu_gemm_static (the emulated GEMM with its scratch in a static device array, allocating nothing)
against the existing entry point emu_gemm_ws with a caller workspace.  Collected last on purpose:
the static scratch is shared by every call on a device, so these tests also show that it carries no
state over from earlier calls."""
import ctypes
import zlib

import numpy as np
import pytest
import torch

from tests.golden.make_golden import gen_inputs


def _params(kind, r3=0, r4=0, out=0):
    from emugen_b200 import _lib

    nv = kind == "nvfp"
    return _lib.EmuGemmParams(0 if nv else 1, 16 if nv else 32, 4 if nv else 2, r3, r4, out)


def test_static_entry_exported_and_rejects_oversized_problems():
    from emugen_b200 import _lib

    L = _lib.load()
    assert "emu_gemm_static" in _lib.SYMBOLS
    prm = _params("nvfp")
    M = N = K = 4096
    need = L.emu_gemm_workspace_size(M, N, K, ctypes.byref(prm))
    assert need > _lib.STATIC_SCRATCH_BYTES
    # the argument checks come first: NULL tensors are reported exactly as emu_gemm reports them
    st = L.emu_gemm_static(None, None, None, None, M, N, K, M, K // 16, N, K // 16, None, ctypes.byref(prm), None, None)
    st_ref = L.emu_gemm(None, None, None, None, M, N, K, M, K // 16, N, K // 16, None, ctypes.byref(prm), None, None)
    assert st == st_ref == 1  # EMU_ERR_INVALID_ARGUMENT
    assert "NULL" in L.emu_last_error().decode()
    # valid-looking (16-byte aligned, never dereferenced) pointers: the size limit rejects the problem
    # on the host, before anything is enqueued
    host = np.zeros(64, dtype=np.uint8)
    p = (host.ctypes.data + 15) // 16 * 16
    st = L.emu_gemm_static(p, p, p, p, M, N, K, M, K // 16, N, K // 16, None, ctypes.byref(prm), p, None)
    assert st == 8  # EMU_ERR_UNSUPPORTED
    msg = L.emu_last_error().decode()
    assert "needs" in msg and str(need) in msg and str(_lib.STATIC_SCRATCH_BYTES) in msg


def _run(entry, a, b, sfa, sfb, M, N, K, alpha, prm, out_dtype):
    from emugen_b200 import _lib

    L = _lib.load()
    out = torch.empty((M, N), dtype=out_dtype, device="cuda")
    al = None if alpha is None else torch.tensor([alpha], dtype=torch.float32, device="cuda")
    args = [a.data_ptr(), b.data_ptr(), sfa.data_ptr(), sfb.data_ptr(), M, N, K, sfa.shape[0], sfa.shape[1],
            sfb.shape[0], sfb.shape[1], None if al is None else al.data_ptr(), ctypes.byref(prm), out.data_ptr()]
    stream = torch.cuda.current_stream().cuda_stream
    if entry == "static":
        st = L.emu_gemm_static(*args, stream)
    else:
        need = L.emu_gemm_workspace_size(M, N, K, ctypes.byref(prm))
        assert need > 0
        ws = torch.empty(need + 1024, dtype=torch.uint8, device="cuda")
        st = L.emu_gemm_ws(*args, (ws.data_ptr() + 1023) // 1024 * 1024, need, stream)
    assert st == 0, L.emu_last_error().decode()
    torch.cuda.synchronize()
    return out


# A larger NVFP4 problem with NaN block scales (sets the NaN row / column flags in the scratch),
# then a smaller MXFP4 one without: the second call must not see the first call's flags.
CASES = [dict(kind="nvfp", data="raw_nan_scales", M=384, N=320, K=2048, r3=0, r4=1, out=0),
         dict(kind="mxfp", data="normal", M=1024, N=1024, K=1024, r3=1, r4=0, out=1)]


@pytest.mark.gpu
def test_static_matches_workspace_entry_on_two_calls_in_a_row():
    from emugen_b200 import _lib

    L = _lib.load()
    inputs, results = [], []
    for c in CASES:
        rng = np.random.default_rng(zlib.crc32(f"static-{c['kind']}-{c['data']}".encode()))
        a, b, sfa, sfb, alpha = gen_inputs(c, rng)
        t = [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (a, b, sfa, sfb)]
        prm = _params(c["kind"], c["r3"], c["r4"], c["out"])
        assert 0 < L.emu_gemm_workspace_size(c["M"], c["N"], c["K"], ctypes.byref(prm)) <= _lib.STATIC_SCRATCH_BYTES
        inputs.append((t, float(alpha) if c["kind"] == "nvfp" else None, prm))
    # two static calls back to back, then the reference entry point on the same inputs
    for c, (t, alpha, prm) in zip(CASES, inputs):
        dt = torch.bfloat16 if c["out"] == 1 else torch.float16
        results.append(_run("static", *t, c["M"], c["N"], c["K"], alpha, prm, dt))
    for c, (t, alpha, prm), got in zip(CASES, inputs, results):
        dt = torch.bfloat16 if c["out"] == 1 else torch.float16
        ref = _run("ws", *t, c["M"], c["N"], c["K"], alpha, prm, dt)
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), c
    assert torch.isnan(results[0].float()).any()          # the NaN scales reached the output
    assert not torch.isnan(results[1].float()).any()      # ... and did not leak into the next call
