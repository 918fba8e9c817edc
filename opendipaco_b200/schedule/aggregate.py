"""Robust aggregation of buffered pseudo-gradients (reference ``schedule/aggregate.py``).

Direction = coordinate-wise ``mean`` / ``trimmed_mean`` (drop one value per side
when there are >= 3) / ``median`` of the raw contributions; magnitude = the sum of
their weights. A single contribution passes through unchanged (bit-identical).
On CUDA tensors the coordinate-wise combine runs in one kernel (a small sorting
network per coordinate, ``csrc/codec.cu``).
"""

from __future__ import annotations

import torch

AGGREGATES = ("mean", "trimmed_mean", "median")


def check_aggregate(name: str) -> str:
    if name not in AGGREGATES:
        raise ValueError(f"aggregate must be one of {AGGREGATES}, got {name!r}")
    return name


def _combine(stack: torch.Tensor, mode: str) -> torch.Tensor:
    if stack.is_cuda and stack.dtype == torch.float32 and 2 <= stack.shape[0] <= 16:
        from ..ops import codec

        return codec.robust_combine(stack, mode)
    if mode == "median":
        return stack.median(dim=0).values
    if mode == "trimmed_mean" and stack.shape[0] >= 3:
        return stack.sort(dim=0).values[1:-1].mean(dim=0)
    return stack.mean(dim=0)


def robust_delta(contributions, *, aggregate: str = "trimmed_mean"):
    check_aggregate(aggregate)
    wsum = float(sum(w for w, _ in contributions))
    grads = [g for _, g in contributions]
    if len(grads) == 1:
        return list(grads[0]), wsum
    return [_combine(torch.stack([g[i] for g in grads]), aggregate) for i in range(len(grads[0]))], wsum
