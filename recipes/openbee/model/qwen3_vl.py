"""The Qwen3-VL model patches OpenBee uses, under the reference's module path (recipes/openbee/model/qwen3_vl.py)."""

from recipes.qwen3_vl.model.qwen3_vl import calculate_model_flops, patch_qwen3vl_conv3d, patch_qwen3vl_model_flops

__all__ = ["calculate_model_flops", "patch_qwen3vl_conv3d", "patch_qwen3vl_model_flops"]
