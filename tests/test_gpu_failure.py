"""Failure detection of the tensor-core kernel without a GPU fault: a pipeline wait is made to run
out (the test hook withholds the first accumulator-ready signal, under a short wait bound); the
kernel must return, the failure must reach the caller through emu_device_status, and the CUDA
context must stay usable -- the next call is bit-exact again.  The reference raises synchronously
on bad input (nvfp_emulation.cpp:99-106); this is the device-side counterpart."""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden.make_golden import gen_inputs
from tests.golden_cases import nan_equal_mismatches


def _case():
    case = dict(kind="nvfp", data="normal", M=256, N=192, K=1024, r3=0, r4=0, out=0)
    a, b, sfa, sfb, alpha = gen_inputs(case, np.random.default_rng(5))
    return a, b, sfa, sfb, float(alpha)


def _gemm(a, b, sfa, sfb, alpha):
    from emugen_b200 import _lib

    return _lib.gemm(*(torch.from_numpy(x).cuda() for x in (a, b, sfa, sfb)), fmt=0, group_size=16, w_reduce=4,
                     stage3_rounding=0, stage4_rounding=0, alpha=torch.tensor([alpha], device="cuda"), out_mode=0,
                     path="tc")


@pytest.mark.gpu
def test_timed_out_wait_is_reported_and_the_context_survives():
    from emugen_b200 import _lib

    L = _lib.load()
    a, b, sfa, sfb, alpha = _case()
    _lib.device_status()                      # nothing pending from earlier tests
    prev = _lib.set_wait_limit(1 << 20)       # about half a millisecond per wait
    L.emu_test_hold_first_ready(1)
    try:
        _gemm(a, b, sfa, sfb, alpha)
        with pytest.raises(_lib.EmuError) as err:
            _lib.device_status()
        assert err.value.status == _lib.EMU_ERR_TIMEOUT
        assert "pipeline wait ran out" in str(err.value)
        _lib.device_status()                  # the record was cleared by the first query
    finally:
        L.emu_test_hold_first_ready(0)
        _lib.set_wait_limit(prev)
    out = _gemm(a, b, sfa, sfb, alpha)
    _lib.device_status()
    ref = oracle.emul_gemm(a, b, sfa, sfb, scale_fmt=0, group_size=16, w_reduce=4, alpha=alpha)
    bits = out.cpu().view(torch.int16).numpy().view(np.uint16)
    assert nan_equal_mismatches(bits, ref, "float16") == 0
