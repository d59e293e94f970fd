from .packing import build_qwen3_vl_packed_position_ids, prepare_packed_model_inputs
from .qwen3_vl import calculate_model_flops, patch_qwen3vl_conv3d, patch_qwen3vl_model_flops

__all__ = ["build_qwen3_vl_packed_position_ids", "calculate_model_flops", "patch_qwen3vl_conv3d",
           "patch_qwen3vl_model_flops", "prepare_packed_model_inputs"]
