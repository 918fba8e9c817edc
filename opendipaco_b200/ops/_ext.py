"""Loader for the in-tree sm_100a extension ``opendipaco_b200._C``.

There is no fallback: CUDA code paths call :func:`ext`, which raises if the
extension was not built (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``).
"""

from __future__ import annotations

import importlib

import torch

_mod = None
_err: dict[int, torch.Tensor] = {}


def ext():
    global _mod
    if _mod is None:
        try:
            _mod = importlib.import_module("opendipaco_b200._C")
        except ImportError as exc:  # pragma: no cover - exercised on misconfigured boxes
            raise RuntimeError(
                "opendipaco_b200._C (the sm_100a kernels) is not built; run "
                "`python setup.py build_ext --inplace` in the repository root") from exc
    return _mod


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def err_word(device) -> torch.Tensor:
    """Per-device int32 error word the kernels' bounded waits write into."""
    d = torch.device(device)
    idx = d.index if d.index is not None else torch.cuda.current_device()
    if idx not in _err:
        _err[idx] = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
    return _err[idx]


class KernelTimeout(RuntimeError):
    """A device-side bounded wait ran out (the kernel returned early)."""


_CODES = {1: "TMA stage never filled", 2: "stage never freed", 3: "accumulator never ready",
          4: "TMEM never released", 5: "peer flag never arrived", 6: "bad arguments"}


def check_errors(device=None) -> None:
    """Raise :class:`KernelTimeout` if any kernel on ``device`` recorded an error."""
    devs = [torch.device(device).index if device is not None else None]
    for idx, t in _err.items():
        if devs[0] is not None and idx != devs[0]:
            continue
        code = int(t.item())
        if code:
            t.zero_()
            raise KernelTimeout(f"cuda:{idx}: device wait timed out ({_CODES.get(code, code)})")
