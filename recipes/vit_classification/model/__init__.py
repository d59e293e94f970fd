from .vit import build_vit_model

__all__ = ["build_vit_model"]
