from .vit_classification_engine import ViTClassificationEngine

__all__ = ["ViTClassificationEngine"]
