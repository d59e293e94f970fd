from recipes.vit_classification.dataset.sampler import InfiniteDistributedSampler

from .dataset import FakeAutoregressiveDataset, build_dataset

__all__ = ["FakeAutoregressiveDataset", "InfiniteDistributedSampler", "build_dataset"]
