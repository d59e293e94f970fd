from .minimal_vlm_engine import MinimalVLMEngine

__all__ = ["MinimalVLMEngine"]
