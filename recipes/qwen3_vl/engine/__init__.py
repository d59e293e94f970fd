from .qwen3_vl_engine import Qwen3VLEngine

__all__ = ["Qwen3VLEngine"]
