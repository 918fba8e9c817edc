"""opendipaco_b200 -- a DiPaCo / DiLoCo training framework built for NVIDIA B200.

Public API parity with OpenDiPaCo (``src/opendipaco/__init__.py``)::

    from opendipaco_b200 import (BackboneConfig, DiPaCoConfig, DiLoCoConfig, PathTopology,
                                 LocalBackend, DiPaCoEngine)

On CUDA devices the engine runs the fused sm_100a executor (flat device buffers,
hand-written tcgen05 GEMMs, attention, RMSNorm, fused cross-entropy, fused
AdamW / 8-bit Adam, one-kernel outer step; NVLink peer-memory outer step across
GPUs). On CPU it runs PyTorch modules and is the numerical oracle.
"""

from .checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
from .config import BackboneConfig, DiLoCoConfig, DiPaCoConfig, SegmentSpec
from .em import assign_paths_by_loss, fit_discriminative_router, path_losses, reshard_by_loss
from .models import PathModel, build_module_bank, build_path_model, warm_start_modules
from .parallel import LocalBackend, SyncBackend, gather_full_bank
from .topology import PathTopology, Segment, Sharing
from .train import DiPaCoEngine, ExecOptions, RoundMetrics

__all__ = [
    "BackboneConfig", "DiPaCoConfig", "DiLoCoConfig", "SegmentSpec", "Segment", "Sharing",
    "PathTopology", "PathModel", "build_module_bank", "build_path_model", "SyncBackend",
    "LocalBackend", "DiPaCoEngine", "ExecOptions", "RoundMetrics", "warm_start_modules",
    "path_losses", "assign_paths_by_loss", "reshard_by_loss", "fit_discriminative_router",
    "gather_full_bank", "save_checkpoint", "load_checkpoint", "latest_checkpoint",
    "AsyncScheduler",
]

try:
    from .parallel import TorchDistBackend  # noqa: F401

    __all__.append("TorchDistBackend")
except Exception:  # pragma: no cover
    pass


def __getattr__(name):
    if name == "AsyncScheduler":
        from .schedule.scheduler import AsyncScheduler

        return AsyncScheduler
    raise AttributeError(name)


__version__ = "0.1.0"
