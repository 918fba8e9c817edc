"""Routing kernels (``csrc/routing.cu``): k-means assignment and bag-of-tokens features."""

from __future__ import annotations

import torch

from ._ext import ext


def kmeans_assign(x: torch.Tensor, centroids: torch.Tensor, k: int = 1) -> torch.Tensor:
    """[N, k] indices of the k nearest centroids (nearest first)."""
    return ext().kmeans_assign(x, centroids, k, False)[0]


def sq_dists(x: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    """[N, K] squared Euclidean distances."""
    return ext().kmeans_assign(x, centroids, 1, True)[1]


def bag_of_tokens(prefixes: list[torch.Tensor], projection: torch.Tensor, vocab_size: int) -> torch.Tensor:
    lens = torch.tensor([0] + [int(p.numel()) for p in prefixes], dtype=torch.long)
    offs = torch.cumsum(lens, 0).to(projection.device)
    ids = (torch.cat([p.reshape(-1).to(torch.int32) for p in prefixes]) if len(prefixes)
           else torch.zeros(0, dtype=torch.int32)).to(projection.device)
    if ids.numel() == 0:
        ids = torch.zeros(1, dtype=torch.int32, device=projection.device)
    return ext().bag_of_tokens(ids, offs, projection.contiguous())
