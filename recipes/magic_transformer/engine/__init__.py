from .magic_transformer_engine import MagicTransformerEngine

__all__ = ["MagicTransformerEngine"]
