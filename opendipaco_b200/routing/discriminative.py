"""Discriminative router: a linear classifier from prefix features to path index.

Trained on (features of a document's prefix, path the document was assigned to) pairs
with full-batch Adam (lr 1e-2, weight decay 1e-4) for a fixed number of epochs. With
``val_fraction > 0`` a seeded random split is held out and the parameters with the lowest
held-out cross-entropy seen during training are kept (early stopping without a patience
parameter). Hyper-parameters and behaviour follow the reference's
``src/opendipaco/routing/discriminative.py``.
"""

from __future__ import annotations

import torch
from torch import nn
from torch.nn.functional import cross_entropy


def _holdout(n: int, fraction: float, seed: int):
    """(train indices, held-out indices or None)."""
    if fraction <= 0 or n < 2:
        return torch.arange(n), None
    order = torch.randperm(n, generator=torch.Generator().manual_seed(seed))
    cut = max(1, int(n * fraction))
    return order[cut:], order[:cut]


class _BestSnapshot:
    """Keeps a copy of a module's state whenever its score improves."""

    def __init__(self):
        self.score, self.state = float("inf"), None

    def offer(self, score: float, module: nn.Module) -> None:
        if score < self.score:
            self.score = score
            self.state = {k: v.detach().clone() for k, v in module.state_dict().items()}

    def restore(self, module: nn.Module) -> None:
        if self.state is not None:
            module.load_state_dict(self.state)


class DiscriminativeRouter(nn.Module):
    def __init__(self, feature_dim: int, num_paths: int):
        super().__init__()
        self.linear = nn.Linear(feature_dim, num_paths)

    def forward(self, features: torch.Tensor) -> torch.Tensor:
        return self.linear(features)

    def fit(self, features: torch.Tensor, labels: torch.Tensor, epochs: int = 200, lr: float = 1e-2,
            weight_decay: float = 1e-4, val_fraction: float = 0.0, seed: int = 0) -> "DiscriminativeRouter":
        train, held = _holdout(features.size(0), val_fraction, seed)
        x, y = features[train], labels[train]
        opt = torch.optim.Adam(self.parameters(), lr=lr, weight_decay=weight_decay)
        best = _BestSnapshot()
        for _ in range(epochs):
            opt.zero_grad()
            cross_entropy(self(x), y).backward()
            opt.step()
            if held is not None:
                with torch.no_grad():
                    best.offer(float(cross_entropy(self(features[held]), labels[held])), self)
        best.restore(self)
        return self

    @torch.no_grad()
    def predict(self, features: torch.Tensor) -> torch.Tensor:
        return self(features).argmax(dim=-1)

    @torch.no_grad()
    def predict_topk(self, features: torch.Tensor, k: int) -> torch.Tensor:
        scores = self(features)
        return scores.topk(min(k, scores.size(-1)), dim=-1).indices
