import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
REF = ROOT / "baseline" / "_ref"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built extension")
    config.addinivalue_line("markers", "multigpu: needs >= 2 GPUs")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture
def reference_pkg():
    """The unmodified reference package installed under baseline/_ref (the oracle)."""
    if not (REF / "opendipaco").is_dir():
        pytest.skip("reference not installed in baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import opendipaco

    return opendipaco


def pytest_collection_modifyitems(config, items):
    # a GPU test on a machine without CUDA is skipped rather than failed
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords or "multigpu" in it.keywords:
            it.add_marker(skip)


os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
