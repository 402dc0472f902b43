"""Loader for the compiled sm_100a extension (``fak_b200._C``).

The extension is built in-tree (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``).  There is no eager/PyTorch fallback for the
kernels: on a CUDA machine a missing extension is an error, never a silent
slow path.
"""
from __future__ import annotations

import importlib

_C = None
_ERR: Exception | None = None


def ext():
    global _C, _ERR
    if _C is not None:
        return _C
    try:
        _C = importlib.import_module("fak_b200._C")
    except ImportError as e:  # pragma: no cover - exercised only without a build
        _ERR = e
        raise ImportError(
            "fak_b200._C (sm_100a kernels) is not built: run `python setup.py build_ext --inplace` "
            f"in the repository root ({e})") from e
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except ImportError:
        return False
