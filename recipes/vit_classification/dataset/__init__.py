from .imagenet import GaussianImageDataset, build_dataset, build_transforms
from .sampler import InfiniteDistributedSampler

__all__ = ["GaussianImageDataset", "InfiniteDistributedSampler", "build_dataset", "build_transforms"]
