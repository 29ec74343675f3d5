"""Process-wide freeze of lazy resolution.

The kernels are compiled ahead of time, but a runtime still resolves things
lazily: loading the extension, allocating alignment and gather scratch, building
multicast state.  A serving engine warms all of that, then freezes; anything that
would still be resolved afterwards raises instead of stalling a decode step
(reference behaviour: ``sparknet/oneshot/_freeze.py:22-58``).  No heavy imports,
so CPU-only tools can import the package.
"""

from __future__ import annotations

import threading

_lock = threading.Lock()
_frozen = False
_reason: str | None = None


class KernelResolutionFrozenError(RuntimeError):
    """Raised when something would be resolved lazily after the freeze."""


def freeze_kernel_resolution(reason: str | None = None) -> None:
    """Refuse every later lazy resolution; call after the serving warm-up."""
    global _frozen, _reason
    with _lock:
        _frozen, _reason = True, reason


def thaw_kernel_resolution() -> None:
    """Allow lazy resolution again (tests and tooling)."""
    global _frozen, _reason
    with _lock:
        _frozen, _reason = False, None


def kernel_resolution_frozen() -> bool:
    """Whether lazy kernel or scratch resolution is refused at the moment."""
    with _lock:
        return _frozen


def raise_if_kernel_resolution_frozen(kind: str, *, target: object | None = None,
                                      cache_key: object | None = None) -> None:
    """Raise KernelResolutionFrozenError, naming ``kind`` and the target, while resolution is frozen."""
    with _lock:
        frozen, reason = _frozen, _reason
    if not frozen:
        return
    parts = [f"sparknet resolution is frozen; refusing {kind}"]
    if target is not None:
        parts.append(f"target={type(target).__name__}")
    if cache_key is not None:
        parts.append(f"key={cache_key!r}")
    if reason is not None:
        parts.append(f"reason={reason}")
    parts.append("prepare it before freezing")
    raise KernelResolutionFrozenError("; ".join(parts))


__all__ = ["KernelResolutionFrozenError", "freeze_kernel_resolution", "kernel_resolution_frozen",
           "raise_if_kernel_resolution_frozen", "thaw_kernel_resolution"]
