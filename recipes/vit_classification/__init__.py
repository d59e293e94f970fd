"""ViT image-classification recipe."""
