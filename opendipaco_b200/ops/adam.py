"""Optimizer kernels (``csrc/adam.cu``): grad-norm clip coefficient, AdamW, 8-bit Adam."""

from __future__ import annotations

import math

import torch

from ._ext import ext

SQ_ELEMS_PER_BLOCK = 1 << 16


def sched_row(lr: float, b1: float, b2: float, step: int, active: bool = True) -> list[float]:
    """[lr, lr / (1 - b1^t), sqrt(1 - b2^t), active] for step t (1-based)."""
    return [lr, lr / (1 - b1 ** step), math.sqrt(1 - b2 ** step), 1.0 if active else 0.0]


def sched_tensor(lr: float, b1: float, b2: float, step: int, device, groups: int = 1) -> torch.Tensor:
    return torch.tensor([sched_row(lr, b1, b2, step)] * groups, dtype=torch.float32, device=device)


def clip_coef(grads: torch.Tensor, P: int, stride: int, G: int, max_norm: float | None,
              work: torch.Tensor | None = None, coef: torch.Tensor | None = None,
              norm_out: torch.Tensor | None = None) -> torch.Tensor:
    nblk = (P + SQ_ELEMS_PER_BLOCK - 1) // SQ_ELEMS_PER_BLOCK
    if work is None:
        work = torch.empty(G * nblk, device=grads.device, dtype=torch.float32)
    if coef is None:
        coef = torch.empty(G, device=grads.device, dtype=torch.float32)
    ext().grad_clip_coef(grads, P, stride, G, float(max_norm or 0.0), work, coef, norm_out, None, 0, 4, 0)
    return coef


def adamw(p, g, m, v, p16, P, stride, stride16, G, coef, sched, b1, b2, eps, wd):
    ext().adamw_step(p, g, m, v, p16, P, stride, stride16, G, coef, sched, b1, b2, eps, wd, None, 0, 4, 0)


def adam8bit_step(p: torch.Tensor, grad: torch.Tensor, st: dict, *, lr, b1, b2, eps, wd, bc1, bc2_sqrt,
                  first: bool, coef=None, p16=None, blocks_per_group: int = 0) -> None:
    """One 8-bit AdamW update of ``p`` in place (state layout of :class:`Adam8bit`)."""
    sched = torch.tensor([lr, lr / bc1, bc2_sqrt, 1.0], dtype=torch.float32, device=p.device)
    ext().adam8bit_step(p.data.reshape(-1), grad.reshape(-1).float().contiguous(), st["m_q"], st["m_absmax"],
                        st["v_q"], st["v_lo"], st["v_scale"], coef, sched, b1, b2, eps, wd, first, p16,
                        blocks_per_group)
