from .prepare import prepare_packed_model_inputs

__all__ = ["prepare_packed_model_inputs"]
