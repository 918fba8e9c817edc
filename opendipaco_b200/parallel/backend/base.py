"""The engine's only communication seam (reference ``src/opendipaco/backend/base.py``).

``global_reduce(key, ReducedDelta)`` combines this node's weighted-summed
pseudo-gradient for module ``key`` with every other node sharing it.
Backends may additionally implement :meth:`SyncBackend.fused_outer_step`, which
the B200 engine prefers: one device-side call that reduces, applies Nesterov and
writes the new globals back into every sharer's working copies.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass

import torch

from ...topology import Path, PathTopology


@dataclass
class ReducedDelta:
    summed: list[torch.Tensor]
    weight: float


class SyncBackend(ABC):
    topology: PathTopology
    rank: int = 0
    world_size: int = 1

    @abstractmethod
    def owned_paths(self) -> list[Path]: ...

    def rank_of_path(self, path: Path) -> int:
        return 0

    @abstractmethod
    def owns_module(self, key: str) -> bool: ...

    @abstractmethod
    def global_reduce(self, key: str, local: ReducedDelta) -> ReducedDelta: ...

    def barrier(self) -> None:
        pass

    def sharing_ranks(self, key: str) -> list[int]:
        """Sorted ranks owning >= 1 path through ``key``."""
        return sorted({self.rank_of_path(p) for p in self.topology.paths_through_module(key)})
