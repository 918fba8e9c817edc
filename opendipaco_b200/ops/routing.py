"""Routing kernels (``csrc/routing.cu``): k-means assignment on the tensor cores, the
deterministic centroid update and bag-of-tokens features."""

from __future__ import annotations

import torch

from ._ext import err_word, ext


def _rows32(t: torch.Tensor) -> torch.Tensor:
    """fp32, contiguous, feature dim padded with zeros to a multiple of 32 (padding
    changes no dot product or norm)."""
    t = t.float().contiguous()
    pad = (-t.size(1)) % 32
    if pad:
        t = torch.nn.functional.pad(t, (0, pad))
    return t


def assign(x: torch.Tensor, centroids: torch.Tensor, k: int = 1, *, want_min: bool = False,
           want_dist: bool = False) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
    """([N, k] nearest centroids, nearest first; [N] nearest squared distance or None;
    [N, K] squared distances or None)."""
    xf, cf = _rows32(x), _rows32(centroids.to(x.device))
    idx, mind, dist = ext().kmeans_assign(xf, cf, k, want_min, want_dist, err_word(x.device))
    return idx, (mind if want_min else None), (dist if want_dist else None)


def kmeans_assign(x: torch.Tensor, centroids: torch.Tensor, k: int = 1) -> torch.Tensor:
    """[N, k] indices of the k nearest centroids (nearest first)."""
    return assign(x, centroids, k)[0]


def sq_dists(x: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    """[N, K] squared Euclidean distances (|x|^2 - 2 x.c + |c|^2, fp32 quality)."""
    return assign(x, centroids, 1, want_dist=True)[2]


def cluster_sums(x: torch.Tensor, idx: torch.Tensor, num_clusters: int) -> tuple[torch.Tensor, torch.Tensor]:
    """([K, D] sums of the rows assigned to each cluster by idx[:, 0], [K] counts);
    fixed summation order, reproducible bit for bit."""
    return ext().kmeans_cluster_sums(x.float().contiguous(), idx.contiguous(), num_clusters)


def bag_of_tokens(prefixes: list[torch.Tensor], projection: torch.Tensor, vocab_size: int) -> torch.Tensor:
    lens = torch.tensor([0] + [int(p.numel()) for p in prefixes], dtype=torch.long)
    offs = torch.cumsum(lens, 0).to(projection.device)
    ids = (torch.cat([p.reshape(-1).to(torch.int32) for p in prefixes]) if len(prefixes)
           else torch.zeros(0, dtype=torch.int32)).to(projection.device)
    if ids.numel() == 0:
        ids = torch.zeros(1, dtype=torch.int32, device=projection.device)
    return ext().bag_of_tokens(ids, offs, projection.contiguous())
