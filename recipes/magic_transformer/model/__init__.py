from .magic_transformer import MagicTransformer, TransformerConfig, build_magic_transformer_model

__all__ = ["MagicTransformer", "TransformerConfig", "build_magic_transformer_model"]
