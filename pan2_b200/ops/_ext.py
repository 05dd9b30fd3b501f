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
        return _CountingProxy(_C) if _COUNTING["on"] else _C
    if _ERR is None:
        try:
            import torch  # noqa: F401  (loads libc10 before the extension)
            _C = importlib.import_module("pan2_b200._C")
            return _CountingProxy(_C) if _COUNTING["on"] else _C
        except ImportError as exc:  # pragma: no cover - depends on the build
            _ERR = exc
    raise RuntimeError(
        "pan2_b200._C (the sm_100a kernels) is not built; run `python setup.py build_ext --inplace`"
    ) from _ERR


# kernels launched by one call of each binding (for the benchmark's launch count)
KERNELS_PER_CALL = {
    "ln_modulate_bwd": 2, "gate_bwd": 2, "mse_fwd": 2, "attn_bwd": 3, "error_flag": 0,
}
_COUNTING = {"on": False, "launches": 0, "by_name": {}}


class _CountingProxy:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn) or not _COUNTING["on"]:
            return fn

        def wrapped(*a, **k):
            n = KERNELS_PER_CALL.get(name, 1)
            _COUNTING["launches"] += n
            _COUNTING["by_name"][name] = _COUNTING["by_name"].get(name, 0) + n
            return fn(*a, **k)
        return wrapped


def start_launch_count() -> None:
    _COUNTING.update(on=True, launches=0, by_name={})


def stop_launch_count() -> dict:
    _COUNTING["on"] = False
    return dict(total=_COUNTING["launches"], by_name=dict(_COUNTING["by_name"]))


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
