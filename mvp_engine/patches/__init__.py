"""Idempotent runtime patches (reference: mvp_engine/patches/registry.py:27-64)."""

from .registry import PatchResult, apply_all_patches, register_patch

__all__ = ["PatchResult", "apply_all_patches", "register_patch"]
