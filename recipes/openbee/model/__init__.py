"""OpenBee uses the Qwen3-VL recipe's model patches and packing helpers unchanged."""

from recipes.qwen3_vl.model import (build_qwen3_vl_packed_position_ids, calculate_model_flops,
                                    patch_qwen3vl_conv3d, patch_qwen3vl_model_flops, prepare_packed_model_inputs)

__all__ = ["build_qwen3_vl_packed_position_ids", "calculate_model_flops", "patch_qwen3vl_conv3d",
           "patch_qwen3vl_model_flops", "prepare_packed_model_inputs"]
