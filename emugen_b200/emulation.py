"""Drop-in for the reference Python engine ``search.emulation`` (search/emulation/*.py).

Mirrors ``RoundStrategy`` / ``coerce_round_strategy`` (rounding.py:10-34), ``HardwareConfig``
(config.py:10-81), ``SearchNVFPEmulationState`` + ``emulate_nvfp_scaled_fp4_mm`` (gemm.py:16-69),
``MMAEngine.emulation_scaled_fp4_mm`` (core.py:69-148) and ``EmulationKernel`` /
``emulated_fp4_mm`` (kernel.py:12-112).  The arithmetic runs in libemugen.so on the GPU and is bit
for bit the reference's for the two element formats the reference quantisers produce:
  group_size 16 -> NVFP4 (E4M3 scales as torch.float8_e4m3fn, f32 scale product),
  group_size 32 -> MXFP4 (UE8M0 scales as uint8, f64 scale product).
The reference lets a caller pass ``unpack_fp4`` / ``linearize_block_scales`` callables
(core.py:85-101).  The kernels read the packed bytes and swizzled scales themselves, so a callable
is accepted only when it computes the standard format of the element type chosen by ``group_size``
-- as the reference's own helpers do, which its callers pass (gemm_compare/backends/mxfp.py:139-144,
search/w3.py:139-150): e2m1 nibbles low first, and the 128x4 swizzled scales decoded as E4M3
(group 16) or 2^(u - 127) (group 32).  Each callable is checked once, on a small probe input;
any other callable raises NotImplementedError instead of being silently ignored.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Callable, Optional

import torch

from . import _lib


class RoundStrategy(Enum):
    """Same members and values as the reference enum (search/emulation/rounding.py:10-16)."""
    RZ = "round_toward_zero"
    RNE = "round_to_nearest_even"
    RU = "round_up"
    RD = "round_down"
    RNA = "round_to_nearest_away"


def coerce_round_strategy(rounding) -> RoundStrategy:
    """Accept RoundStrategy (this one or the reference's, matched by name) or 0=RZ / 1=RNE."""
    if isinstance(rounding, RoundStrategy):
        return rounding
    name = getattr(rounding, "name", None)
    if isinstance(name, str) and name in RoundStrategy.__members__ and isinstance(rounding, Enum):
        return RoundStrategy[name]
    if rounding == 0:
        return RoundStrategy.RZ
    if rounding == 1:
        return RoundStrategy.RNE
    raise TypeError(f"Rounding must be RoundStrategy or nvfp_cpp_emul code (RZ=0, RNE=1), got {rounding!r}")


def _rounding_code(rounding) -> int:
    r = coerce_round_strategy(rounding)
    if r == RoundStrategy.RZ:
        return _lib.EMU_RZ
    if r == RoundStrategy.RNE:
        return _lib.EMU_RNE
    raise NotImplementedError(f"Rounding {r} not implemented in to_float32_with_rounding")


@dataclass
class HardwareConfig:
    """Accumulator configuration (reference config.py:10-81).  w_stage3 / w_stage4 are validated
    and carried but change no result, exactly as in the reference (core.py:31-38)."""
    w_stage3: int = 34
    w_stage4: int = 28
    w_reduce: int = 4
    stage3_rounding: RoundStrategy = RoundStrategy.RZ
    stage4_rounding: RoundStrategy = RoundStrategy.RZ
    name: str = "custom"
    description: str = ""

    def __post_init__(self):
        if self.w_stage3 < 20 or self.w_stage3 > 50:
            raise ValueError(f"w_stage3 should be in [20, 50], got {self.w_stage3}")
        if self.w_stage4 < 20 or self.w_stage4 > 50:
            raise ValueError(f"w_stage4 should be in [20, 50], got {self.w_stage4}")
        if self.w_reduce < 2 or self.w_reduce > 16:
            raise ValueError(f"w_reduce should be in [2, 16], got {self.w_reduce}")

    @classmethod
    def for_rtx_5090(cls) -> "HardwareConfig":
        return cls(w_stage3=34, w_stage4=28, w_reduce=4, stage3_rounding=RoundStrategy.RZ,
                   stage4_rounding=RoundStrategy.RZ, name="RTX_5090",
                   description="NVIDIA RTX 5090 with NVFP4 input, FP16 output")

    @classmethod
    def from_dict(cls, d: dict) -> "HardwareConfig":
        d = dict(d)
        d.setdefault("w_reduce", 4)
        for k in ("stage3_rounding", "stage4_rounding"):
            if k in d and isinstance(d[k], str):
                d[k] = RoundStrategy[d[k]]
        return cls(**d)

    def to_dict(self) -> dict:
        return {"w_stage3": self.w_stage3, "w_stage4": self.w_stage4, "w_reduce": self.w_reduce,
                "stage3_rounding": self.stage3_rounding.name, "stage4_rounding": self.stage4_rounding.name,
                "name": self.name, "description": self.description}


CONFIG_RTX_5090 = HardwareConfig.for_rtx_5090()


_E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)
_helper_verdicts: dict = {}


def _probe_unpack(fn) -> bool:
    """Does fn(packed [R, K/2] uint8, (R, K)) unpack e2m1 nibbles, low nibble first?"""
    packed = torch.arange(256, dtype=torch.int32).to(torch.uint8).reshape(16, 16)
    lut = torch.tensor(_E2M1)
    want = torch.stack([lut[(packed & 15).long()], lut[(packed >> 4).long()]], dim=-1).reshape(16, 32)
    got = fn(packed, (16, 32))
    return tuple(got.shape) == (16, 32) and bool((got.float().cpu() == want).all())


def _probe_linearize(fn, group_size: int) -> bool:
    """Does fn(swizzled [128, 4] scales, 128, 4) decode the 128x4 swizzled layout to [128, 4] f32
    values, E4M3 for group 16, 2^(u - 127) for group 32?"""
    rows, cols = 128, 4
    lin = (torch.arange(rows * cols, dtype=torch.int64).reshape(rows, cols) * 37 + 11) % 120 + 1  # no NaN codes
    swz = torch.empty(rows * cols, dtype=torch.uint8)
    r = torch.arange(rows).reshape(-1, 1)
    c = torch.arange(cols).reshape(1, -1)
    off = (r % 32) * 16 + (r // 32) * 4 + c   # one 128-row, 4-column tile of the swizzled layout
    swz[off.reshape(-1)] = lin.reshape(-1).to(torch.uint8)
    swz = swz.reshape(rows, cols)
    if group_size == 16:
        arg, want = swz.view(torch.float8_e4m3fn), lin.to(torch.uint8).view(torch.float8_e4m3fn).float()
    else:
        arg, want = swz, torch.exp2(lin.float() - 127.0)
    got = fn(arg, rows, cols)
    return tuple(got.shape) == (rows, cols) and bool((got.float().cpu() == want).all())


def _check_helpers(unpack_fp4, linearize_block_scales, group_size: int) -> None:
    """Raise unless every given callable computes the standard format (module docstring)."""
    for fn, kind in ((unpack_fp4, "unpack_fp4"), (linearize_block_scales, "linearize_block_scales")):
        if fn is None:
            continue
        key = (fn, kind, group_size)
        if key not in _helper_verdicts:
            try:
                ok = _probe_unpack(fn) if kind == "unpack_fp4" else _probe_linearize(fn, group_size)
            except Exception:  # a callable that cannot run on the probe is not the standard one either
                ok = False
            _helper_verdicts[key] = ok
        if not _helper_verdicts[key]:
            raise NotImplementedError(
                f"{kind}={getattr(fn, '__name__', fn)!r} does not compute the standard "
                f"{'NVFP4' if group_size == 16 else 'MXFP4'} format; the emulation kernels read packed e2m1 "
                f"bytes and 128x4 swizzled scales directly and cannot apply a custom {kind}")


class MMAEngine:
    """Reference ``MMAEngine`` (core.py:53-148), computed by libemugen.so."""

    @staticmethod
    def emulation_scaled_fp4_mm(a_fp4, b_fp4, scale_a, scale_b, alpha_tensor, M, N, K, W_stage3=25, W_stage4=25,
                                w_reduce=4, stage3_rounding=RoundStrategy.RZ, stage4_rounding=RoundStrategy.RZ,
                                m_chunk_size=128, group_size: int = 16,
                                unpack_fp4: Optional[Callable] = None,
                                linearize_block_scales: Optional[Callable] = None,
                                out_mode: int = _lib.EMU_OUT_F16) -> torch.Tensor:
        """Scaled FP4 MMA emulation -> fp16 [M, N] (or f32 / bf16 via ``out_mode``)."""
        r3 = _rounding_code(stage3_rounding)
        r4 = _rounding_code(stage4_rounding)
        assert K % group_size == 0, f"K must be multiple of group_size ({group_size})"
        G = K // group_size
        assert G % w_reduce == 0, f"G=K/group_size ({G}) must be divisible by w_reduce ({w_reduce})"
        if int(m_chunk_size) <= 0:
            raise ValueError("m_chunk_size must be positive")
        if a_fp4.shape[0] != M or b_fp4.shape[0] != N or a_fp4.shape[1] * 2 != K:
            raise ValueError(f"tensor shapes {tuple(a_fp4.shape)}, {tuple(b_fp4.shape)} do not match M={M} N={N} K={K}")
        if group_size == 16:
            fmt = _lib.EMU_FMT_NVFP4
        elif group_size == 32:
            fmt = _lib.EMU_FMT_MXFP4
        else:
            raise NotImplementedError(f"group_size {group_size}: only 16 (NVFP4) and 32 (MXFP4) are supported")
        _check_helpers(unpack_fp4, linearize_block_scales, group_size)
        return _lib.gemm(a_fp4, b_fp4, scale_a, scale_b, fmt=fmt, group_size=group_size, w_reduce=int(w_reduce),
                         stage3_rounding=r3, stage4_rounding=r4, alpha=alpha_tensor, out_mode=out_mode)


@dataclass
class SearchNVFPEmulationState:
    """Quantized tensors + emulation knobs (reference gemm.py:16-32)."""
    a_fp4: torch.Tensor
    b_fp4: torch.Tensor
    scale_a: torch.Tensor
    scale_b: torch.Tensor
    alpha: torch.Tensor
    out_dtype: torch.dtype
    w_stage3: int
    w_stage4: int
    w_reduce: int
    group_size: int
    m_chunk_size: int
    stage3_rounding: RoundStrategy | int
    stage4_rounding: RoundStrategy | int


def emulate_nvfp_scaled_fp4_mm(state, *, unpack_fp4: Optional[Callable] = None,
                               linearize_block_scales: Optional[Callable] = None) -> torch.Tensor:
    """Reference gemm.py:35-69: MMAEngine on ``state`` then ``.to(state.out_dtype)``.  bf16 output is
    bf16(fp16(x)) exactly like the reference; it is produced in one pass by the kernel."""
    M = state.a_fp4.shape[0]
    N = state.b_fp4.shape[0]
    K = state.a_fp4.shape[1] * 2
    od = state.out_dtype
    out_mode = _lib.EMU_OUT_BF16_VIA_F16 if od == torch.bfloat16 else _lib.EMU_OUT_F16
    out = MMAEngine.emulation_scaled_fp4_mm(
        state.a_fp4, state.b_fp4, state.scale_a, state.scale_b, state.alpha, M, N, K,
        W_stage3=state.w_stage3, W_stage4=state.w_stage4, w_reduce=state.w_reduce,
        stage3_rounding=state.stage3_rounding, stage4_rounding=state.stage4_rounding,
        m_chunk_size=state.m_chunk_size, group_size=state.group_size, unpack_fp4=unpack_fp4,
        linearize_block_scales=linearize_block_scales, out_mode=out_mode)
    return out if out.dtype == od else out.to(od)


class EmulationKernel:
    """Reference kernel.py:12-96: NVFP4 (group 16) emulation with a fixed accumulator config."""

    def __init__(self, config: Optional[HardwareConfig] = None, w_stage3: int = 34, w_stage4: int = 28,
                 w_reduce: int = 4, stage3_rounding=RoundStrategy.RZ, stage4_rounding=RoundStrategy.RZ,
                 m_chunk_size: int = 128):
        if config is not None:
            w_stage3, w_stage4, w_reduce = config.w_stage3, config.w_stage4, config.w_reduce
            stage3_rounding, stage4_rounding = config.stage3_rounding, config.stage4_rounding
        self.w_stage3, self.w_stage4, self.w_reduce = w_stage3, w_stage4, w_reduce
        self.stage3_rounding, self.stage4_rounding = stage3_rounding, stage4_rounding
        self.m_chunk_size = m_chunk_size

    def __call__(self, a, b, block_scale_a, block_scale_b, alpha, out_dtype=torch.float16):
        return self.forward(a, b, block_scale_a, block_scale_b, alpha, out_dtype)

    def forward(self, a, b, block_scale_a, block_scale_b, alpha, out_dtype=torch.float16):
        M, N, K = a.shape[0], b.shape[0], a.shape[1] * 2
        out_mode = _lib.EMU_OUT_BF16_VIA_F16 if out_dtype == torch.bfloat16 else _lib.EMU_OUT_F16
        res = MMAEngine.emulation_scaled_fp4_mm(
            a, b, block_scale_a, block_scale_b, alpha, M, N, K, W_stage3=self.w_stage3, W_stage4=self.w_stage4,
            w_reduce=self.w_reduce, stage3_rounding=self.stage3_rounding, stage4_rounding=self.stage4_rounding,
            m_chunk_size=self.m_chunk_size, group_size=16, out_mode=out_mode)
        return res if res.dtype == out_dtype else res.to(out_dtype)

    @classmethod
    def for_rtx_5090(cls) -> "EmulationKernel":
        return cls(w_stage3=34, w_stage4=28, w_reduce=4, stage3_rounding=RoundStrategy.RZ,
                   stage4_rounding=RoundStrategy.RZ)

    @classmethod
    def from_config(cls, config: HardwareConfig) -> "EmulationKernel":
        return cls(config=config)


def emulated_fp4_mm(a, b, block_scale_a, block_scale_b, alpha, out_dtype=torch.float16,
                    config: Optional[HardwareConfig] = None) -> torch.Tensor:
    kernel = EmulationKernel.from_config(config) if config else EmulationKernel.for_rtx_5090()
    return kernel(a, b, block_scale_a, block_scale_b, alpha, out_dtype)


emulated_scaled_fp4_mm = emulated_fp4_mm


@dataclass(frozen=True)
class AccumModel:
    """Accumulator model for sweeps (no reference counterpart: the reference accepts w_stage3 /
    w_stage4 and ignores them, core.py:31-38).  align3 / align4: alignment widths of stage 3 /
    stage 4 (0 = exact, the reference); align_rounding: RoundStrategy.RZ truncates the aligned
    addends, RNE rounds them to nearest even; order: stage-3 f64 order when align3 == 0
    (0 left to right = reference, 1 right to left, 2 pairwise tree).  Semantics in include/emugen.h."""
    align3: int = 0
    align4: int = 0
    align_rounding: RoundStrategy | int = RoundStrategy.RZ
    order: int = 0


def emulate_with_model(state, model: AccumModel) -> torch.Tensor:
    """``emulate_nvfp_scaled_fp4_mm(state)`` under ``model`` (all-zero model = identical results)."""
    od = state.out_dtype
    out_mode = _lib.EMU_OUT_BF16_VIA_F16 if od == torch.bfloat16 else _lib.EMU_OUT_F16
    gs = int(state.group_size)
    if gs not in (16, 32):
        raise NotImplementedError(f"group_size {gs}: only 16 (NVFP4) and 32 (MXFP4) are supported")
    out = _lib.gemm_model(state.a_fp4, state.b_fp4, state.scale_a, state.scale_b,
                          fmt=_lib.EMU_FMT_NVFP4 if gs == 16 else _lib.EMU_FMT_MXFP4, group_size=gs,
                          w_reduce=int(state.w_reduce), stage3_rounding=_rounding_code(state.stage3_rounding),
                          stage4_rounding=_rounding_code(state.stage4_rounding), alpha=state.alpha,
                          out_mode=out_mode, align3=int(model.align3), align4=int(model.align4),
                          align_rounding=_rounding_code(model.align_rounding), order=int(model.order))
    return out if out.dtype == od else out.to(od)

__all__ = ["RoundStrategy", "coerce_round_strategy", "HardwareConfig", "CONFIG_RTX_5090", "MMAEngine",
           "SearchNVFPEmulationState", "emulate_nvfp_scaled_fp4_mm", "EmulationKernel", "emulated_fp4_mm",
           "emulated_scaled_fp4_mm", "AccumModel", "emulate_with_model"]
