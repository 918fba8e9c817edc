"""Generative k-means router (cluster i -> path i).

Reference: ``src/opendipaco/routing/kmeans.py:12-55``: init = ``randperm`` of the
points with a seeded generator; loop: distances -> argmin -> per-cluster mean (an
empty cluster is re-seeded to the point farthest from its nearest centroid) ->
stop when the centroid shift norm < ``tol``.

On CUDA features the assignment step (``|x|^2 - 2 x.c + |c|^2``, argmin / top-k)
runs in one sm_100a kernel and the centroid update is a deterministic ordered
segmented mean (no float atomics), so the fit is reproducible run to run.
"""

from __future__ import annotations

import torch


class KMeansRouter:
    def __init__(self, num_paths: int, max_iters: int = 50, seed: int = 0, tol: float = 1e-4):
        self.num_paths = num_paths
        self.max_iters = max_iters
        self.seed = seed
        self.tol = tol
        self.centroids: torch.Tensor | None = None

    @staticmethod
    def _dists(x: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
        if x.is_cuda:
            from ..ops import routing as K

            return K.sq_dists(x, c).clamp_min_(0).sqrt_()
        return torch.cdist(x, c)

    def fit(self, features: torch.Tensor) -> "KMeansRouter":
        n = features.size(0)
        if n < self.num_paths:
            raise ValueError(f"need >= {self.num_paths} samples to fit, got {n}")
        gen = torch.Generator(device=features.device).manual_seed(self.seed)
        idx = torch.randperm(n, generator=gen, device=features.device)[: self.num_paths]
        cent = features[idx].clone()
        for _ in range(self.max_iters):
            d = self._dists(features, cent)
            assign = d.argmin(dim=1)
            new = cent.clone()
            for k in range(self.num_paths):
                m = assign == k
                if m.any():
                    new[k] = features[m].mean(dim=0)
                else:
                    new[k] = features[d.min(dim=1).values.argmax()]
            shift = (new - cent).norm()
            cent = new
            if shift < self.tol:
                break
        self.centroids = cent
        return self

    def predict(self, features: torch.Tensor) -> torch.Tensor:
        if self.centroids is None:
            raise RuntimeError("KMeansRouter must be fit() before predict()")
        if features.is_cuda:
            from ..ops import routing as K

            return K.kmeans_assign(features, self.centroids.to(features.device), 1)[:, 0]
        return torch.cdist(features, self.centroids.to(features.device)).argmin(dim=1)

    def predict_topk(self, features: torch.Tensor, k: int) -> torch.Tensor:
        if self.centroids is None:
            raise RuntimeError("KMeansRouter must be fit() before predict_topk()")
        k = min(k, self.centroids.size(0))
        if features.is_cuda:
            from ..ops import routing as K

            return K.kmeans_assign(features, self.centroids.to(features.device), k)
        d = torch.cdist(features, self.centroids.to(features.device))
        return d.topk(k, largest=False, dim=1).indices
