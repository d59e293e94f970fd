"""Packed 3-D M-RoPE positions, under the reference's module path (recipes/openbee/model/packing/qwen3_vl.py)."""

from recipes.qwen3_vl.model.packing.qwen3_vl import build_qwen3_vl_packed_position_ids

__all__ = ["build_qwen3_vl_packed_position_ids"]
