"""Loader of the in-tree sm_100a extension (``oscar_b200/_C*.so``).

The extension is built by ``python setup.py build_ext --inplace`` (or
``__graft_entry__.build()``).  On a machine with a GPU every op requires it and
fails loudly if it is missing; CPU tensors use the pure-torch reference path.
"""
from __future__ import annotations

import importlib

from ..utils import launches as _launches

# launches per binding call (all others launch exactly one kernel)
_MULTI = {"num_sms": 0, "argmax": 2}
_EXT = None
_ERR: Exception | None = None


class _Counted:
    """Proxy that counts kernel launches of the extension's entry points."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        n = _MULTI.get(name, 1)

        def call(*a, **k):
            _launches.add(n)
            return fn(*a, **k)

        setattr(self, name, call)
        return call


def ext():
    """Return the compiled extension module, raising a clear error if unavailable."""
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            _EXT = _Counted(importlib.import_module("oscar_b200._C"))
        except Exception as e:  # pragma: no cover - depends on the build
            _ERR = e
    if _EXT is None:
        raise RuntimeError(
            "oscar_b200 CUDA extension is not built (run `python setup.py build_ext --inplace`): "
            f"{_ERR!r}")
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
