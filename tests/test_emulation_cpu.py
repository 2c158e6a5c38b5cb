"""Host logic of the search.emulation drop-in (no GPU): custom unpack / scale-linearisation callables
are accepted only when they compute the standard format (search/emulation/core.py:85-101 lets a
caller pass them; the kernels read packed bytes and swizzled scales directly)."""
import pytest
import torch

from emugen_b200 import emulation

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def std_unpack(packed, shape):
    lo, hi = (packed & 15).long(), (packed >> 4).long()
    return E2M1[torch.stack([lo, hi], dim=-1)].reshape(shape).half()


def _unswizzle(sw, rows, cols):
    r = torch.arange(rows).reshape(-1, 1)
    c = torch.arange(cols).reshape(1, -1)
    kt = sw.shape[1] // 4
    off = (r // 128) * kt * 512 + (c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4
    return sw.reshape(-1)[off]


def std_linearize_e4m3(sw, rows, cols):
    return _unswizzle(sw.view(torch.uint8), rows, cols).view(torch.float8_e4m3fn).float()


def std_linearize_ue8m0(sw, rows, cols):
    return torch.exp2(_unswizzle(sw.view(torch.uint8), rows, cols).float() - 127.0)


def test_standard_helpers_pass_the_check():
    emulation._check_helpers(std_unpack, std_linearize_e4m3, 16)
    emulation._check_helpers(std_unpack, std_linearize_ue8m0, 32)
    emulation._check_helpers(None, None, 16)


@pytest.mark.parametrize("unpack,linearize,gs", [
    (lambda p, s: std_unpack(p, s).flip(-1), None, 16),                       # high nibble first
    (lambda p, s: std_unpack(p, s).abs(), None, 32),                          # sign dropped
    (None, std_linearize_ue8m0, 16),                                          # UE8M0 decode for NVFP4
    (None, std_linearize_e4m3, 32),                                           # E4M3 decode for MXFP4
    (None, lambda sw, r, c: sw.view(torch.uint8)[:r, :c].float(), 32),        # swizzle ignored
    (None, lambda sw, r, c: 1 / 0, 16),                                       # cannot run at all
])
def test_custom_helpers_raise(unpack, linearize, gs):
    with pytest.raises(NotImplementedError, match="standard"):
        emulation._check_helpers(unpack, linearize, gs)
