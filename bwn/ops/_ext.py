"""Loader for the in-tree native extension ``bwn._C``.

The extension registers ``torch.ops.bwn.*``.  CUDA tensors always go to the
extension; if it is missing on a machine with a GPU, :func:`require` raises
instead of falling back to PyTorch, so a test can never pass on a silent
eager path.
"""
from __future__ import annotations

import importlib
import os

import torch

_C = None
_err: Exception | None = None


def load():
    global _C, _err
    if _C is not None or _err is not None:
        return _C
    try:
        _C = importlib.import_module("bwn._C")
    except Exception as e:  # noqa: BLE001 - report the real import error later
        _err = e
    return _C


def available() -> bool:
    return load() is not None


def require():
    if load() is None:
        here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        raise RuntimeError(
            "bwn CUDA extension is not built (import bwn._C failed: %r). Build it in-tree with "
            "`python setup.py build_ext --inplace` in %s" % (_err, here)
        )
    return _C


def ops():
    require()
    return torch.ops.bwn


def status() -> int:
    """Device error-status word (bit flags set by kernels that gave up a bounded wait)."""
    if load() is None or not torch.cuda.is_available():
        return 0
    return int(_C.status())


def status_clear() -> None:
    if load() is not None and torch.cuda.is_available():
        _C.status_clear()


def check_status(where: str = "") -> None:
    s = status()
    if s:
        status_clear()
        names = {1: "mbarrier wait timeout", 2: "peer wait timeout", 4: "bounds check", 8: "bad argument",
                 16: "flag wait timeout"}
        what = ", ".join(v for k, v in names.items() if s & k)
        raise RuntimeError(f"bwn kernel reported an error ({what}; status=0x{s:x}) {where}")
