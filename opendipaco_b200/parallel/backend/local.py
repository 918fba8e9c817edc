"""Single-process backend: every path is local, ``global_reduce`` is the identity.

Reference ``src/opendipaco/backend/local.py``. This is the correctness oracle and
the single-GPU configuration.
"""

from __future__ import annotations

from ...topology import Path, PathTopology
from .base import ReducedDelta, SyncBackend


class LocalBackend(SyncBackend):
    def __init__(self, topology: PathTopology):
        self.topology = topology

    def owned_paths(self) -> list[Path]:
        return self.topology.paths()

    def owns_module(self, key: str) -> bool:
        return True

    def global_reduce(self, key: str, local: ReducedDelta) -> ReducedDelta:
        return local
