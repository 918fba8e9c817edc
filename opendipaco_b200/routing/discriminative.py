"""Test-time linear router over prefix features (reference ``routing/discriminative.py``).

Adam (lr 1e-2, wd 1e-4), 200 full-batch epochs; with ``val_fraction > 0`` a seeded
held-out split keeps the parameters with the lowest held-out loss.
"""

from __future__ import annotations

import torch
from torch import nn


class DiscriminativeRouter(nn.Module):
    def __init__(self, feature_dim: int, num_paths: int):
        super().__init__()
        self.linear = nn.Linear(feature_dim, num_paths)

    def forward(self, features: torch.Tensor) -> torch.Tensor:
        return self.linear(features)

    def fit(self, features: torch.Tensor, labels: torch.Tensor, epochs: int = 200,
            lr: float = 1e-2, weight_decay: float = 1e-4, val_fraction: float = 0.0,
            seed: int = 0) -> "DiscriminativeRouter":
        opt = torch.optim.Adam(self.parameters(), lr=lr, weight_decay=weight_decay)
        ce = nn.functional.cross_entropy
        if val_fraction <= 0 or features.size(0) < 2:
            for _ in range(epochs):
                opt.zero_grad()
                ce(self(features), labels).backward()
                opt.step()
            return self
        n = features.size(0)
        perm = torch.randperm(n, generator=torch.Generator().manual_seed(seed))
        nv = max(1, int(n * val_fraction))
        vi, ti = perm[:nv], perm[nv:]
        best, state = float("inf"), None
        for _ in range(epochs):
            opt.zero_grad()
            ce(self(features[ti]), labels[ti]).backward()
            opt.step()
            with torch.no_grad():
                v = float(ce(self(features[vi]), labels[vi]))
            if v < best:
                best, state = v, {k: t.detach().clone() for k, t in self.state_dict().items()}
        if state is not None:
            self.load_state_dict(state)
        return self

    @torch.no_grad()
    def predict(self, features: torch.Tensor) -> torch.Tensor:
        return self(features).argmax(dim=-1)

    @torch.no_grad()
    def predict_topk(self, features: torch.Tensor, k: int) -> torch.Tensor:
        logits = self(features)
        return logits.topk(min(k, logits.size(-1)), dim=-1).indices
