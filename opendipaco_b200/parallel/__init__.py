from .backend import LocalBackend, ReducedDelta, SyncBackend
from .gather import gather_full_bank
from .placement import block_sizes, path_ranks, rank_paths

__all__ = ["LocalBackend", "ReducedDelta", "SyncBackend", "gather_full_bank", "block_sizes",
           "path_ranks", "rank_paths"]
try:
    from .backend import TorchDistBackend  # noqa: F401

    __all__.append("TorchDistBackend")
except Exception:  # pragma: no cover
    pass
