"""Kernel-patch kit (reference: mvp_engine/kit/model/liger.py:33-142).

The reference swaps module-level symbols of HF model files for Liger's
Triton kernels before model construction.  This engine's models already run
native sm_100a kernels, and Triton is not used on any hot path, so the
``official`` route reports that nothing needs patching.  The ``custom`` route
is kept: a ``LigerPatch`` replaces ``module.attr`` with any callable (for
example one of ``mvp_engine.ops``), which is how third-party model code can be
pointed at the engine's kernels.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from typing import Any, Callable


@dataclass(frozen=True)
class LigerPatch:
    module: str
    attr: str
    replacement: Callable[..., Any] | Any


@dataclass(frozen=True)
class LigerKernelReport:
    route: str
    applied: list[str] = field(default_factory=list)
    skipped: list[str] = field(default_factory=list)
    excluded: list[str] = field(default_factory=list)


class LigerKernelKit:
    def apply(self, *, family: str | None = None, modules: str | dict[str, bool] = "all",
              custom_patches: list[LigerPatch] | None = None, exclude: list[str] | None = None) -> LigerKernelReport:
        excluded = set(exclude or ["cross_entropy", "fused_linear_cross_entropy"])
        if custom_patches:
            applied, skipped = [], []
            for p in custom_patches:
                name = f"{p.module}.{p.attr}"
                if p.attr in excluded:
                    skipped.append(name)
                    continue
                mod = importlib.import_module(p.module)
                if not hasattr(mod, p.attr):
                    raise AttributeError(f"{p.module} has no attribute {p.attr!r}")
                setattr(mod, p.attr, p.replacement)
                applied.append(name)
            return LigerKernelReport("custom", applied, skipped, sorted(excluded))
        names = list(modules) if isinstance(modules, dict) else ([] if modules == "all" else [modules])
        return LigerKernelReport("official", [], [f"{family}:{n}" for n in names] or [f"{family}:all"],
                                 sorted(excluded))
