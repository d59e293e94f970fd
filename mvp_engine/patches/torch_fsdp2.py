"""Mixed-precision input casting for torch FSDP2 modules recomputed under activation checkpointing
(reference behaviour: mvp_engine/patches/torch_fsdp2.py:44-118).

When an FSDP2-sharded module runs inside ``torch.utils.checkpoint`` and its recompute happens in the
backward, ``FSDPState._pre_forward`` sees the state ``PRE_BACKWARD`` and returns the inputs as they are:
the ``MixedPrecisionPolicy`` cast of floating-point inputs to ``param_dtype`` is skipped, so the recomputed
forward gets fp32 inputs against bf16 parameters (a dtype error, or activations whose metadata differ from
the ones saved in the forward).  torch 2.11 still behaves this way (``tests/test_patches_cpu.py``
reproduces it on CPU).

The patch wraps ``_pre_forward``: after the original returns, if the state is still ``PRE_BACKWARD`` (the
early-return path) and the policy casts forward inputs, floating-point tensors in ``args`` / ``kwargs`` are
cast to ``param_dtype``.  On a torch that already casts there, the extra cast finds nothing to change.
It touches only torch's FSDP2 backend (``parallel.backend_kwargs.impl: torch``); the native runtime does
not use ``FSDPState``.
"""

from __future__ import annotations

import functools
import importlib
from types import ModuleType
from typing import Any, Optional

import torch
from torch.utils._pytree import tree_map

from .types import PatchResult

PATCH_NAME = "torch_fsdp2_checkpoint_recompute_cast"
_MARK = "_mvp_recompute_cast"
_STATE_MODULES = ("torch.distributed.fsdp._fully_shard._fsdp_state", "torch.distributed._composable.fsdp._fsdp_state")


def _state_module() -> Optional[ModuleType]:
    for name in _STATE_MODULES:
        try:
            return importlib.import_module(name)
        except ImportError:
            continue
    return None


def _cast_floats(tree: Any, dtype: torch.dtype) -> Any:
    def cast(x: Any) -> Any:
        if isinstance(x, torch.Tensor) and x.is_floating_point() and x.dtype != dtype:
            return x.to(dtype)
        return x

    return tree_map(cast, tree)


def apply_fsdp2_checkpoint_recompute_cast_patch(fsdp_state: Optional[ModuleType] = None) -> PatchResult:
    """Install the wrapper on ``fsdp_state.FSDPState`` (torch's module by default); idempotent."""
    mod = fsdp_state if fsdp_state is not None else _state_module()
    if mod is None:
        return PatchResult(PATCH_NAME, "skipped", "this torch has no FSDP2 state module")
    state_cls = getattr(mod, "FSDPState", None)
    training = getattr(mod, "TrainingState", None)
    original = getattr(state_cls, "_pre_forward", None) if state_cls is not None else None
    if original is None or training is None or not hasattr(training, "PRE_BACKWARD"):
        return PatchResult(PATCH_NAME, "skipped", "FSDPState._pre_forward / TrainingState.PRE_BACKWARD not found")
    if getattr(original, _MARK, False):
        return PatchResult(PATCH_NAME, "skipped", "already applied")
    recompute_state = training.PRE_BACKWARD

    @functools.wraps(original)
    def _pre_forward(self, module, args, kwargs):
        args, kwargs = original(self, module, args, kwargs)
        if self._training_state == recompute_state:  # the early return taken by checkpoint recompute
            policy = getattr(self, "_mp_policy", None)
            dtype = getattr(policy, "param_dtype", None)
            if dtype is not None and getattr(policy, "cast_forward_inputs", False):
                args, kwargs = _cast_floats(args, dtype), _cast_floats(kwargs, dtype)
        return args, kwargs

    setattr(_pre_forward, _MARK, True)
    state_cls._pre_forward = _pre_forward
    return PatchResult(PATCH_NAME, "applied", "inputs of recomputed FSDP2 modules are cast to param_dtype")
