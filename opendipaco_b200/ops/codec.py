"""GPU codec kernels (``csrc/codec.cu``): int4 / int8 quantisation, decode, robust combine."""

from __future__ import annotations

import torch

from ._ext import ext

_MODES = {"mean": 0, "trimmed_mean": 1, "median": 2}


def quant_int4(x: torch.Tensor, want_resid: bool = True):
    """-> (packed uint8 [ngroups*64], scale fp32 [ngroups], residual or None)."""
    p, s, r = ext().quant_int4(x.float().contiguous(), want_resid)
    return p, s, (r if want_resid else None)


def dequant_int4(packed: torch.Tensor, scale: torch.Tensor, n: int, g: int = 128, out=None,
                 weight: float = 1.0, accumulate: bool = False) -> torch.Tensor:
    if out is None:
        out = torch.empty(n, device=packed.device, dtype=torch.float32)
    ext().dequant_int4(packed.contiguous(), scale.float().contiguous(), n, g, out, weight, accumulate)
    return out


def quant_int8(x: torch.Tensor, want_resid: bool = True):
    """-> (q int8, scale as a python float = absmax / 127, residual or None)."""
    q, amax, r = ext().quant_int8(x.float().contiguous(), want_resid)
    return q, float(amax.item()) / 127.0, (r if want_resid else None)


def robust_combine(stack: torch.Tensor, mode: str) -> torch.Tensor:
    return ext().robust_combine(stack, _MODES[mode])
