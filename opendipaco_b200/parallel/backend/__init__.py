from .base import ReducedDelta, SyncBackend
from .local import LocalBackend

__all__ = ["SyncBackend", "ReducedDelta", "LocalBackend"]
try:
    from .torch_dist import TorchDistBackend  # noqa: F401

    __all__.append("TorchDistBackend")
except Exception:  # pragma: no cover
    pass
