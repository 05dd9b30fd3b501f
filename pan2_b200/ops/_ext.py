"""Loader for the compiled sm_100a extension ``pan2_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``).  Every CUDA tensor path in :mod:`pan2_b200.ops` goes through it; when
a CUDA tensor reaches an op and the extension is missing, the op raises instead of falling back to
a PyTorch implementation.
"""
from __future__ import annotations

import importlib

_C = None
_ERR = None


def ext():
    """Return the loaded ``pan2_b200._C`` module or raise with the import error."""
    global _C, _ERR
    if _C is not None:
        return _C
    if _ERR is None:
        try:
            _C = importlib.import_module("pan2_b200._C")
            return _C
        except ImportError as exc:  # pragma: no cover - depends on the build
            _ERR = exc
    raise RuntimeError(
        "pan2_b200._C (the sm_100a kernels) is not built; run `python setup.py build_ext --inplace`"
    ) from _ERR


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
