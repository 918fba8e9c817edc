"""Cross-entropy kernels over bf16 logits (``csrc/loss.cu``)."""

from __future__ import annotations

import torch

from ._ext import ext


def cross_entropy_rows(logits: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Per-row ``lse - logit[target]`` (0 where target < 0), fp32."""
    x = logits if logits.stride(-1) == 1 else logits.contiguous()
    x = x.reshape(-1, x.shape[-1])
    if x.stride(0) < x.shape[1]:
        x = x.contiguous()
    return ext().cross_entropy_rows(x, target.reshape(-1))


def cross_entropy_sum(logits: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    return cross_entropy_rows(logits, target).sum()
