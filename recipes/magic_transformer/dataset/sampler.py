"""The infinite distributed sampler, under the reference's module path (recipes/magic_transformer/dataset/sampler.py);
the implementation is shared with the ViT recipe."""

from recipes.vit_classification.dataset.sampler import InfiniteDistributedSampler

__all__ = ["InfiniteDistributedSampler"]
