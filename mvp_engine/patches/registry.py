"""Registry of process-wide runtime patches (reference: mvp_engine/patches/registry.py:27-64).

A patch is a callable returning a :class:`PatchResult`; it must be idempotent and skip itself (status
``skipped``, with the reason) on library versions it does not recognise.  :func:`apply_all_patches` runs
every registered patch once per process: ``MVP_ENGINE_DISABLE_RUNTIME_PATCHES=1`` turns them all off, and
``MVP_ENGINE_STRICT_RUNTIME_PATCHES=1`` makes a patch that raises an error instead of a warning.  The
launcher and the torch FSDP2 backend call it; both calls after the first return the recorded results.
"""

from __future__ import annotations

import os
import warnings
from typing import Callable

from .torch_fsdp2 import PATCH_NAME as _FSDP2_RECOMPUTE_CAST, apply_fsdp2_checkpoint_recompute_cast_patch
from .types import PatchResult

PatchFn = Callable[[], PatchResult]

_PATCHES: list[tuple[str, PatchFn]] = [(_FSDP2_RECOMPUTE_CAST, apply_fsdp2_checkpoint_recompute_cast_patch)]
_RESULTS: dict[str, PatchResult] = {}


def register_patch(name: str) -> Callable[[PatchFn], PatchFn]:
    """Decorator adding a patch to the registry (applied by the next :func:`apply_all_patches`)."""

    def deco(fn: PatchFn) -> PatchFn:
        _PATCHES.append((name, fn))
        return fn

    return deco


def _flag(var: str) -> bool:
    return os.environ.get(var, "").strip().lower() in ("1", "true", "yes", "on")


def apply_all_patches() -> list[PatchResult]:
    """Apply every registered patch not applied yet in this process; returns one result per patch."""
    if _flag("MVP_ENGINE_DISABLE_RUNTIME_PATCHES"):
        return [PatchResult("runtime_patches", "skipped", "disabled by MVP_ENGINE_DISABLE_RUNTIME_PATCHES")]
    strict = _flag("MVP_ENGINE_STRICT_RUNTIME_PATCHES")
    for name, fn in _PATCHES:
        if name in _RESULTS:
            continue
        try:
            _RESULTS[name] = fn()
        except Exception as exc:
            if strict:
                raise RuntimeError(f"runtime patch {name} failed: {exc}") from exc
            _RESULTS[name] = PatchResult(name, "failed", str(exc))
            warnings.warn(f"runtime patch {name!r} failed: {exc}", RuntimeWarning, stacklevel=2)
    return [_RESULTS[name] for name, _ in _PATCHES]
