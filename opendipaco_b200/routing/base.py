"""Routing protocols and the deterministic bag-of-tokens featurizer.

Reference: ``src/opendipaco/routing/base.py:18-64``. DiPaCo routes whole documents
by a feature of their prefix. ``BagOfTokensFeaturizer`` = normalised token
histogram -> fixed seeded N(0, 1/d) projection -> L2 normalise. Its projection is
drawn from ``torch.Generator().manual_seed(seed)`` exactly as the reference does,
so shard specs built by either framework route identically.

On CUDA inputs (``device='cuda'``) the histogram x projection runs as one sm_100a
kernel (``opendipaco_b200/csrc/routing.cu``): each CTA walks one prefix's tokens
and accumulates projection rows (a sparse-count x dense GEMV), then normalises.
"""

from __future__ import annotations

from typing import Protocol, runtime_checkable

import torch


@runtime_checkable
class Featurizer(Protocol):
    feature_dim: int

    def __call__(self, prefixes: list[torch.Tensor]) -> torch.Tensor: ...


@runtime_checkable
class Router(Protocol):
    def predict(self, features: torch.Tensor) -> torch.Tensor: ...


class BagOfTokensFeaturizer:
    def __init__(self, vocab_size: int, feature_dim: int = 256, seed: int = 0,
                 device: str | torch.device = "cpu"):
        self.vocab_size = vocab_size
        self.feature_dim = feature_dim
        gen = torch.Generator().manual_seed(seed)
        self.projection = torch.randn(vocab_size, feature_dim, generator=gen) / feature_dim ** 0.5
        self.device = torch.device(device)
        self._proj_dev = None

    def __call__(self, prefixes: list[torch.Tensor]) -> torch.Tensor:
        if self.device.type == "cuda":
            from ..ops import routing as K

            if self._proj_dev is None:
                self._proj_dev = self.projection.to(self.device)
            return K.bag_of_tokens(prefixes, self._proj_dev, self.vocab_size).cpu()
        # normalised counts @ projection == mean of the projection rows of the prefix
        # tokens: gather the rows and take a per-prefix segment mean (no dense counts).
        lens = torch.tensor([int(p.numel()) for p in prefixes], dtype=torch.long)
        feats = torch.zeros(len(prefixes), self.feature_dim)
        if lens.sum() > 0:
            ids = torch.cat([p.reshape(-1).long() for p in prefixes]).clamp(max=self.vocab_size - 1)
            seg = torch.repeat_interleave(torch.arange(len(prefixes)), lens)
            feats.index_add_(0, seg, self.projection[ids])
            feats /= lens.clamp(min=1).unsqueeze(1).float()
        return torch.nn.functional.normalize(feats, dim=-1)
