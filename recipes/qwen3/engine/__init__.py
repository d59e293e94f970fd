from .qwen3_engine import Qwen3Engine

__all__ = ["Qwen3Engine"]
