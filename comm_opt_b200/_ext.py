"""Loader of the native extension ``comm_opt_b200._C`` (sm_100a kernels).

The extension is built in-tree (``python setup.py build_ext --inplace``). On a machine with a GPU a
missing or stale extension is an error, never a silent fallback: every op of this package that
runs on the GPU goes through ``native()``.
"""
from __future__ import annotations

import importlib

_mod = None
_err: Exception | None = None


def native():
    """Return the ``_C`` module or raise ``RuntimeError`` explaining how to build it."""
    global _mod, _err
    if _mod is not None:
        return _mod
    try:
        _mod = importlib.import_module("comm_opt_b200._C")
    except Exception as e:  # pragma: no cover - exercised only without a build
        _err = e
        raise RuntimeError(
            "comm_opt_b200 native extension is not built or failed to load "
            f"({type(e).__name__}: {e}); run `python setup.py build_ext --inplace` at the repo root"
        ) from e
    return _mod


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False
