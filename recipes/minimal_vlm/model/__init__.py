from .qwen3_vl import apply_freeze_policy, build_qwen3_vl_model

__all__ = ["apply_freeze_policy", "build_qwen3_vl_model"]
