"""Generative k-means router (cluster i -> path i).

Reference: ``src/opendipaco/routing/kmeans.py:12-55``: init = ``randperm`` of the
points with a seeded generator; loop: distances -> argmin -> per-cluster mean (an
empty cluster is re-seeded to the point farthest from its nearest centroid) ->
stop when the centroid shift norm < ``tol``.

On CUDA features every iteration runs on the device with no per-cluster host loop:
the assignment (``|x|^2 - 2 x.c + |c|^2`` with x.c on the tensor cores, argmin / top-k
fused into the epilogue) is one kernel, the per-cluster sums another (ordered, no float
atomics, so the fit is reproducible run to run), and the mean, the re-seeding of empty
clusters and the shift are a few tensor ops. The only host sync per iteration is the
convergence test, as in the reference.
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

    def fit(self, features: torch.Tensor) -> "KMeansRouter":
        n = features.size(0)
        if n < self.num_paths:
            raise ValueError(f"need >= {self.num_paths} samples to fit, got {n}")
        gen = torch.Generator(device=features.device).manual_seed(self.seed)
        idx = torch.randperm(n, generator=gen, device=features.device)[: self.num_paths]
        cent = features[idx].clone()
        if features.is_cuda:
            self.centroids = self._fit_device(features.float().contiguous(), cent.float())
            return self
        for _ in range(self.max_iters):
            d = torch.cdist(features, cent)
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

    def _fit_device(self, x: torch.Tensor, cent: torch.Tensor) -> torch.Tensor:
        from ..ops import routing as K

        for _ in range(self.max_iters):
            idx, mind, _ = K.assign(x, cent, 1, want_min=True)
            sums, counts = K.cluster_sums(x, idx, self.num_paths)
            mean = sums / counts.clamp_min(1).unsqueeze(1).float()
            # an empty cluster takes the point farthest from its nearest centroid
            far = x[mind.argmax()]
            new = torch.where((counts == 0).unsqueeze(1), far.unsqueeze(0), mean)
            shift = (new - cent).norm()
            cent = new
            if shift < self.tol:
                break
        return cent

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
