from .packing import prepare_packed_model_inputs
from .qwen3 import calculate_model_flops, patch_qwen3_model_flops

__all__ = ["calculate_model_flops", "patch_qwen3_model_flops", "prepare_packed_model_inputs"]
