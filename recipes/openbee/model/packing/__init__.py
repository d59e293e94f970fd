from .prepare import build_packed_fa2_varlen_kwargs, build_qwen3_vl_packed_position_ids, prepare_packed_model_inputs

__all__ = ["build_packed_fa2_varlen_kwargs", "build_qwen3_vl_packed_position_ids", "prepare_packed_model_inputs"]
