"""Packed-batch preparation, under the reference's module path (recipes/openbee/model/packing/prepare.py)."""

from recipes.qwen3_vl.model.packing.prepare import build_packed_fa2_varlen_kwargs, prepare_packed_model_inputs

from .qwen3_vl import build_qwen3_vl_packed_position_ids

__all__ = ["build_packed_fa2_varlen_kwargs", "build_qwen3_vl_packed_position_ids", "prepare_packed_model_inputs"]
