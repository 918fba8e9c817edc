"""DiLoCo primitives: inner LR schedule, optimizer factories, pseudo-gradients.

Reference: ``src/opendipaco/optim/diloco.py:26-92``.

* inner: AdamW (or blockwise 8-bit Adam), LR = linear warmup then cosine to
  ``inner_lr * inner_min_lr_ratio`` over the whole run; constant when the
  schedule is "constant" or the horizon is unknown.
* outer: SGD with Nesterov momentum (``lr=outer_lr``, ``momentum=outer_momentum``,
  no weight decay) over the authoritative copies of the shared modules, driven by
  the pseudo-gradient ``global - local`` written into ``.grad``.

The B200 engine runs the same outer update inside one fused kernel
(``opendipaco_b200/ops/outer.py``); its math is kept bit-compatible with
``torch.optim.SGD`` in fp32 (first step ``buf = g``; then ``buf = m*buf + g``;
``p -= lr * (g + m*buf)``), and these factories remain the CPU oracle.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from ..config import DiLoCoConfig


def inner_lr_at(step: int, total_steps: int | None, cfg: DiLoCoConfig) -> float:
    peak, warm = cfg.inner_lr, cfg.inner_warmup_steps
    if warm > 0 and step < warm:
        return peak * (step + 1) / warm
    if cfg.inner_lr_schedule == "constant" or total_steps is None:
        return peak
    frac = (step - warm) / max(total_steps - warm, 1)
    frac = min(max(frac, 0.0), 1.0)
    cos = 0.5 * (1.0 + math.cos(math.pi * frac))
    return peak * (cfg.inner_min_lr_ratio + (1.0 - cfg.inner_min_lr_ratio) * cos)


def make_inner_optimizer(model: nn.Module, cfg: DiLoCoConfig) -> torch.optim.Optimizer:
    if getattr(cfg, "optim_8bit", False):
        from .adam8bit import Adam8bit

        return Adam8bit(model.parameters(), lr=cfg.inner_lr, betas=cfg.inner_betas,
                        weight_decay=cfg.inner_weight_decay)
    return torch.optim.AdamW(model.parameters(), lr=cfg.inner_lr, betas=cfg.inner_betas,
                             weight_decay=cfg.inner_weight_decay)


def make_outer_optimizer(modules: dict[str, nn.Module], cfg: DiLoCoConfig) -> torch.optim.Optimizer:
    params = [p for m in modules.values() for p in m.parameters()]
    return torch.optim.SGD(params, lr=cfg.outer_lr, momentum=cfg.outer_momentum,
                           nesterov=cfg.outer_nesterov, weight_decay=0.0)


@torch.no_grad()
def module_delta(global_mod: nn.Module, local_mod: nn.Module) -> list[torch.Tensor]:
    return [g.detach() - l.detach() for g, l in zip(global_mod.parameters(), local_mod.parameters())]


@torch.no_grad()
def apply_outer_grads(global_mod: nn.Module, delta: list[torch.Tensor]) -> None:
    for p, d in zip(global_mod.parameters(), delta):
        p.grad = d.to(p.device, p.dtype)
