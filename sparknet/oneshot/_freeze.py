"""Process-wide gate on lazy set-up work after a serving warm-up.

The kernels here are compiled ahead of time, so nothing is JIT-compiled at run time,
but a runtime still does some work lazily on first use: loading the extension and
allocating its alignment and gather scratch.  A serving engine runs its warm-up,
then closes the gate; any such work that would still happen later raises
``KernelResolutionFrozenError`` instead of allocating inside a decode step or a graph
capture.  The public names and the behaviour match the reference's kernel-resolution
freeze (``sparknet/oneshot/_freeze.py:22-58`` there); the state here is one gate
object that also counts the refusals it issued.  No heavy imports: CPU-only tools
import this package.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field


class KernelResolutionFrozenError(RuntimeError):
    """Lazy set-up (scratch allocation, extension loading) was requested after the gate closed."""


@dataclass
class _Gate:
    closed: bool = False
    why: str | None = None
    refusals: int = 0
    mutex: threading.Lock = field(default_factory=threading.Lock, repr=False)

    def set(self, closed: bool, why: str | None) -> None:
        with self.mutex:
            self.closed, self.why = closed, why

    def snapshot(self) -> tuple[bool, str | None]:
        with self.mutex:
            return self.closed, self.why

    def refuse(self) -> int:
        with self.mutex:
            self.refusals += 1
            return self.refusals


_GATE = _Gate()


def freeze_kernel_resolution(reason: str | None = None) -> None:
    """Close the gate: every later lazy set-up raises.  Call once the warm-up is done."""
    _GATE.set(True, reason)


def thaw_kernel_resolution() -> None:
    """Open the gate again (tests and tooling)."""
    _GATE.set(False, None)


def kernel_resolution_frozen() -> bool:
    """Whether lazy set-up is refused right now."""
    return _GATE.snapshot()[0]


def refused_resolutions() -> int:
    """How many lazy set-ups the gate has refused in this process."""
    with _GATE.mutex:
        return _GATE.refusals


def raise_if_kernel_resolution_frozen(kind: str, *, target: object | None = None,
                                      cache_key: object | None = None) -> None:
    """Raise ``KernelResolutionFrozenError`` if the gate is closed.

    The message names what was asked for (``kind``), the owner's class (``target``),
    the cache key if any, and the reason given when the gate was closed."""
    closed, why = _GATE.snapshot()
    if not closed:
        return
    count = _GATE.refuse()
    subject = kind if target is None else f"{kind} for {type(target).__name__}"
    if cache_key is not None:
        subject += f" (key {cache_key!r})"
    because = f" because {why}" if why else ""
    raise KernelResolutionFrozenError(
        f"sparknet: {subject} was requested after resolution was frozen{because}; "
        f"do it during warm-up, before freeze_kernel_resolution() (refusal #{count})")


__all__ = ["KernelResolutionFrozenError", "freeze_kernel_resolution", "kernel_resolution_frozen",
           "raise_if_kernel_resolution_frozen", "refused_resolutions", "thaw_kernel_resolution"]
