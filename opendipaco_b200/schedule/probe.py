"""Trusted-probe screen against data poisoning (reference ``schedule/probe.py``).

An audit checker measures the path's loss on a small clean probe before and after
the inner steps; the owner rejects the update when it raised the probe loss by more
than ``abs_margin + rel_margin * |before|``. Unmeasurable (non-finite) losses never
block.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from ..train.loop import token_loss_sum


@torch.no_grad()
def probe_loss(model: nn.Module, sequences: torch.Tensor, *, batch_size: int = 8) -> float:
    if sequences is None or sequences.numel() == 0:
        return float("nan")
    if batch_size < 1:
        raise ValueError(f"probe batch_size must be >= 1, got {batch_size}")
    try:
        dev = next(model.parameters()).device
    except StopIteration:
        return float("nan")
    was = model.training
    model.eval()
    try:
        total, n = token_loss_sum(model, sequences, batch_size=batch_size, device=dev)
    finally:
        if was:
            model.train()
    return total / n if n else float("nan")


def is_harmful(before: float, after: float, *, abs_margin: float = 0.05, rel_margin: float = 0.02) -> bool:
    if not (math.isfinite(before) and math.isfinite(after)):
        return False
    return after - before > abs_margin + rel_margin * abs(before)


def as_finite_float(x) -> float | None:
    if isinstance(x, bool) or not isinstance(x, (int, float)):
        return None
    return float(x) if math.isfinite(x) else None


def safe_probe_loss(probe, model: nn.Module) -> float | None:
    try:
        return probe.loss(model)
    except Exception:
        return None


class TrustedProbe:
    def __init__(self, sequences: torch.Tensor | None, *, batch_size: int = 8):
        self.sequences = sequences
        self.batch_size = int(batch_size)

    @property
    def empty(self) -> bool:
        return self.sequences is None or self.sequences.numel() == 0

    def loss(self, model: nn.Module) -> float:
        return probe_loss(model, self.sequences, batch_size=self.batch_size)
