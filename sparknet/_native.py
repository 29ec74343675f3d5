"""Loader for the compiled extension ``sparknet._C``.

The extension is built in place (``python setup.py build_ext --inplace``).  On a
machine with a CUDA device the collectives require it: a missing or stale build
raises instead of falling back to another backend, so no rank silently changes
transport.  On a host without a GPU (the build host) importing this module is
fine; only calling into the extension needs it.
"""

from __future__ import annotations

import importlib

_module = None
_error: Exception | None = None


def load():
    """Return the extension module, raising a descriptive error if it is missing."""
    global _module, _error
    if _module is not None:
        return _module
    try:
        importlib.import_module("torch")  # the extension links libc10 / libtorch: torch loads them
        _module = importlib.import_module("sparknet._C")
    except Exception as exc:  # noqa: BLE001 - re-raised with context below
        _error = exc
        raise RuntimeError(
            "sparknet's native extension is not built or failed to load "
            f"({exc}); run `python setup.py build_ext --inplace` in the repository root"
        ) from exc
    return _module


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def loaded_path() -> str | None:
    """Filesystem path of the loaded extension (for provenance in receipts)."""
    return getattr(_module, "__file__", None) if _module is not None else None
