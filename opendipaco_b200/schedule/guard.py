"""Server-side sanity checks on submitted updates (reference ``schedule/guard.py``).

Non-finite anything (pseudo-gradient, private weights, reported loss) rejects a
contribution; an optional L2 cap clips oversized pseudo-gradients.
"""

from __future__ import annotations

import math

import torch


def all_finite(obj) -> bool:
    if torch.is_tensor(obj):
        return bool(torch.isfinite(obj).all())
    if isinstance(obj, dict):
        return all(all_finite(v) for v in obj.values())
    if isinstance(obj, (list, tuple)):
        return all(all_finite(v) for v in obj)
    return True


def loss_ok(loss, *, empty: bool = False) -> bool:
    if empty or loss is None:
        return True
    try:
        return math.isfinite(float(loss))
    except (TypeError, ValueError):
        return False


def contribution_ok(loss, empty, *tensor_structures) -> bool:
    return loss_ok(loss, empty=bool(empty)) and all(all_finite(s) for s in tensor_structures)


def clip_norm_(tensors, max_norm: float) -> float:
    """Scale ``tensors`` in place to joint L2 norm <= ``max_norm``; return the pre-clip norm."""
    total = math.sqrt(sum(float(t.detach().float().pow(2).sum()) for t in tensors))
    if total > max_norm:
        s = max_norm / (total + 1e-12)
        for t in tensors:
            t.detach().mul_(s)
    return total
