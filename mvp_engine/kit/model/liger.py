"""Kernel-patch kit (public API of the reference's ``mvp_engine/kit/model/liger.py:33-142``).

The reference swaps module-level symbols of HF modelling files for Liger's Triton kernels before a model
is built: either through Liger's ``apply_liger_kernel_to_<family>`` helpers (the official route) or
through an explicit ``{kernel name: LigerPatch}`` map for custom models (the custom route).

On this engine the engine's own model families call hand-written sm_100a kernels directly, and Triton
kernels are not used on a hot path, so:

* the official route for a native family (``qwen3``, ``qwen3_vl``, ``vit``) reports that nothing needs
  patching; for any other family it raises, naming the custom route as the way to point that model at
  this engine's kernels;
* the custom route is the reference's: every enabled ``LigerPatch`` rebinds ``module.attr`` (to an
  ``mvp_engine.ops`` function, typically), before the model is built.

``excluded_modules`` defaults to the loss kernels on both routes: recipes compute token-normalised
losses and need per-token values, which a fused mean-reducing loss does not return.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass
from typing import Any, Literal, Optional

# kernel names the reference accepts in ``modules`` / ``excluded_modules`` / custom patch keys
SUPPORTED_MODULES = frozenset({"rope", "rms_norm", "layer_norm", "swiglu", "geglu", "cross_entropy",
                               "fused_linear_cross_entropy"})
DEFAULT_EXCLUDED_MODULES = ("cross_entropy", "fused_linear_cross_entropy")
# families whose models in this engine already run the native kernels
NATIVE_FAMILIES = frozenset({"qwen3", "qwen3_vl", "vit"})


@dataclass(frozen=True)
class LigerPatch:
    """One symbol swap: ``setattr(importlib.import_module(module), attr, replacement)``."""

    module: str
    attr: str
    replacement: Any


@dataclass(frozen=True)
class LigerKernelReport:
    """What one ``apply`` did: the route, the helper (none here), the kernel switches it acted on and the
    ``module.attr`` symbols it rebound."""

    model_family: Optional[str]
    route: Literal["official", "custom"]
    helper: Optional[str] = None
    applied: Optional[dict[str, bool]] = None
    patched: tuple[str, ...] = ()


def _validate(names, what: str) -> None:
    bad = sorted(set(names) - SUPPORTED_MODULES)
    if bad:
        raise ValueError(f"Unsupported Liger module(s) in {what}: {bad}. Choose from {sorted(SUPPORTED_MODULES)}.")


def _family_of(model_name_or_path: str, trust_remote_code: bool) -> str:
    """``model_type`` of a local HF directory, or the family a preset name of this engine denotes."""
    import json
    import os

    cfg = os.path.join(model_name_or_path, "config.json")
    if os.path.isfile(cfg):
        with open(cfg) as f:
            return str(json.load(f).get("model_type", ""))
    name = model_name_or_path.lower()
    for family in ("qwen3_vl", "qwen3-vl", "qwen3", "vit"):
        if family in name:
            return family.replace("-", "_")
    raise ValueError(f"cannot tell the model family of {model_name_or_path!r}; pass model_family")


class LigerKernelKit:
    def apply(self, model_name_or_path: Optional[str] = None, *, model_family: Optional[str] = None,
              modules: str | dict[str, bool] = "auto", excluded_modules: tuple[str, ...] = DEFAULT_EXCLUDED_MODULES,
              custom_patches: Optional[dict[str, LigerPatch]] = None,
              trust_remote_code: bool = True) -> LigerKernelReport:
        """Rebind kernels before the model is built (see the module docstring for the two routes)."""
        if isinstance(modules, str) and modules != "auto":
            raise ValueError('`modules` must be "auto" or a dict[str, bool].')
        excluded = set(excluded_modules)
        _validate(excluded, "excluded_modules")
        if custom_patches is not None:
            _validate(custom_patches, "custom_patches")
            enabled = sorted(set(custom_patches) - excluded)
            patched = []
            for name in enabled:
                p = custom_patches[name]
                target = importlib.import_module(p.module)
                if not hasattr(target, p.attr):
                    raise AttributeError(f"{p.module!r} has no symbol {p.attr!r} to rebind")
                setattr(target, p.attr, p.replacement)
                patched.append(f"{p.module}.{p.attr}")
            return LigerKernelReport(model_family, "custom", applied=dict.fromkeys(enabled, True),
                                     patched=tuple(patched))
        if isinstance(modules, dict):
            _validate(modules, "modules")
        family = model_family
        if family is None:
            if model_name_or_path is None:
                raise ValueError("Provide model_name_or_path or model_family for the official route.")
            family = _family_of(model_name_or_path, trust_remote_code)
        if family not in NATIVE_FAMILIES:
            raise ValueError(f"no kernel patching for model family {family!r}: this engine's own families "
                             f"({sorted(NATIVE_FAMILIES)}) run native kernels; point another model at "
                             "mvp_engine.ops with custom_patches={name: LigerPatch(module, attr, op)}")
        return LigerKernelReport(family, "official", helper=None, applied={})
