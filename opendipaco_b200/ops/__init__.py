"""Python entry points of the hand-written sm_100a kernels (``opendipaco_b200/csrc``)."""

from ._ext import KernelTimeout, available, check_errors, ext

__all__ = ["ext", "available", "check_errors", "KernelTimeout"]
