"""RMSNorm / embedding kernels (``csrc/norm.cu``) on 2-D (or grouped) tensors."""

from __future__ import annotations

import torch

from ._ext import ext


def rms_norm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float):
    """x: [R, H] fp32 -> (bf16 y [R, H], fp32 rstd [R])."""
    R, H = x.shape
    y = torch.empty(R, H, device=x.device, dtype=torch.bfloat16)
    rstd = torch.empty(R, device=x.device, dtype=torch.float32)
    ext().rmsnorm_fwd(x, 0, w, 0, y, 0, rstd, R, H, 1, eps)
    return y, rstd


def rms_norm_bwd(x, w, rstd, dy, dres=None):
    """Returns (dx fp32 [R, H], dw fp32 [H])."""
    R, H = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(H, device=x.device, dtype=torch.float32)
    nblk = (R + 7) // 8  # room for the kernel's 8-row blocks (used when few rows)
    work = torch.empty(nblk * H, device=x.device, dtype=torch.float32)
    ext().rmsnorm_bwd(x, 0, w, 0, rstd, dy.float().contiguous(), 0, dres, dx, 0, None, dw, 0, work, R, H, 1, 0.0)
    return dx, dw


def embedding_fwd(ids: torch.Tensor, E: torch.Tensor) -> torch.Tensor:
    ids32 = ids.reshape(-1).to(torch.int32)
    R, (V, H) = ids32.numel(), E.shape
    out = torch.empty(R, H, device=E.device, dtype=torch.float32)
    ext().embedding_fwd(ids32, E, 0, out, R, H, 1, V)
    return out.view(*ids.shape, H)


def embedding_bwd(ids: torch.Tensor, dx: torch.Tensor, V: int) -> torch.Tensor:
    ids32 = ids.reshape(-1).to(torch.int32)
    H = dx.shape[-1]
    dE = torch.zeros(V, H, device=dx.device, dtype=torch.float32)
    ext().embedding_bwd(ids32, dx.reshape(-1, H).float().contiguous(), 0, dE, 0, ids32.numel(), H, 1, V)
    return dE
