"""Loader for the in-tree sm_100a extension ``torchtitan_b200/_C*.so``.

On a CUDA tensor every op requires this extension; a missing or stale build
raises instead of silently falling back.  CPU tensors use the plain-PyTorch
restatements in ``ops/reference.py`` (used by CPU tests and gloo runs).
"""
from __future__ import annotations

import importlib

_mod = None
_err: Exception | None = None
_trace_ns = None  # set by ``graph.traceable.traceable_kernels()`` while a step is being traced


def ext():
    global _mod, _err
    if _trace_ns is not None:
        return _trace_ns
    if _mod is None and _err is None:
        try:
            _mod = importlib.import_module("torchtitan_b200._C")
        except Exception as e:  # noqa: BLE001
            _err = e
    if _mod is None:
        raise RuntimeError(
            "torchtitan_b200._C (sm_100a kernels) is not built or failed to load: "
            f"{_err!r}. Build it with `python setup.py build_ext --inplace`."
        )
    return _mod


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
