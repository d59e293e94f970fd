"""Idempotent runtime patches (reference: mvp_engine/patches/registry.py:27-64, patches/types.py,
patches/torch_fsdp2.py)."""

from .registry import apply_all_patches, register_patch
from .torch_fsdp2 import apply_fsdp2_checkpoint_recompute_cast_patch
from .types import PatchResult, PatchStatus

__all__ = ["PatchResult", "PatchStatus", "apply_all_patches", "apply_fsdp2_checkpoint_recompute_cast_patch",
           "register_patch"]
