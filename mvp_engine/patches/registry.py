"""Fail-closed registry of process-wide runtime patches.

Each patch is a callable returning a :class:`PatchResult`; patches apply once
per process.  ``MVP_ENGINE_DISABLE_RUNTIME_PATCHES=1`` skips all of them and
``MVP_ENGINE_STRICT_RUNTIME_PATCHES=1`` turns a failed patch into an error
instead of a warning (reference: mvp_engine/patches/registry.py:27-64,
mvp_engine/patches/types.py:11-17).  The one patch the reference carries
(FSDP2 input casting under activation-checkpoint recompute for older torch)
is a no-op on the torch this engine targets; it is registered as a version
check so the behaviour is explicit.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable

from ..utils.log import simple_info


@dataclass(frozen=True)
class PatchResult:
    name: str
    applied: bool
    reason: str = ""


_PATCHES: list[tuple[str, Callable[[], PatchResult]]] = []
_APPLIED: dict[str, PatchResult] = {}


def register_patch(name: str) -> Callable[[Callable[[], PatchResult]], Callable[[], PatchResult]]:
    def deco(fn: Callable[[], PatchResult]) -> Callable[[], PatchResult]:
        _PATCHES.append((name, fn))
        return fn

    return deco


def _truthy(var: str) -> bool:
    return os.environ.get(var, "0").strip().lower() in ("1", "true", "yes", "on")


def apply_all_patches() -> list[PatchResult]:
    if _truthy("MVP_ENGINE_DISABLE_RUNTIME_PATCHES"):
        return []
    strict = _truthy("MVP_ENGINE_STRICT_RUNTIME_PATCHES")
    out = []
    for name, fn in _PATCHES:
        if name in _APPLIED:
            out.append(_APPLIED[name])
            continue
        try:
            res = fn()
        except Exception as exc:
            if strict:
                raise RuntimeError(f"runtime patch {name} failed: {exc}") from exc
            simple_info(f"runtime patch {name} skipped: {exc}", "warning")
            res = PatchResult(name, False, str(exc))
        _APPLIED[name] = res
        out.append(res)
    return out


@register_patch("torch_fsdp2_recompute_cast")
def _fsdp2_recompute_cast() -> PatchResult:
    import torch

    major, minor = (int(x) for x in torch.__version__.split(".")[:2])
    if (major, minor) >= (2, 9):
        return PatchResult("torch_fsdp2_recompute_cast", False, "not needed on torch >= 2.9")
    return PatchResult("torch_fsdp2_recompute_cast", False, "torch FSDP2 backend only; native runtime unaffected")
