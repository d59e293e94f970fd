"""Model construction from the recipe config, under the reference's module path (recipes/magic_transformer/model/builder.py)."""

from .magic_transformer import build_magic_transformer_model

__all__ = ["build_magic_transformer_model"]
