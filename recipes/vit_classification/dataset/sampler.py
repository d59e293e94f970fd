"""Never-ending rank-sharded sampler (reference: recipes/vit_classification/dataset/sampler.py:10-70).

Each pass over the dataset is a fresh permutation seeded by ``seed + pass``
(or the identity when ``shuffle`` is off), padded by wrapping (or truncated
with ``drop_last``) to a multiple of the replica count; rank r takes every
``num_replicas``-th index starting at r — the ``DistributedSampler`` split,
repeated forever for iteration-based loops.
"""

from __future__ import annotations

import math
from collections.abc import Iterator, Sized

import torch
from torch.utils.data import Sampler


class InfiniteDistributedSampler(Sampler[int]):
    def __init__(self, dataset: Sized, num_replicas: int, rank: int, *, shuffle: bool = True, seed: int = 0,
                 drop_last: bool = False) -> None:
        n = len(dataset)
        if n <= 0:
            raise ValueError("InfiniteDistributedSampler requires a non-empty dataset.")
        if not 0 <= rank < num_replicas:
            raise ValueError(f"rank {rank} outside [0, {num_replicas})")
        self.dataset, self.dataset_size = dataset, n
        self.num_replicas, self.rank = int(num_replicas), int(rank)
        self.shuffle, self.seed, self.drop_last = shuffle, int(seed), drop_last
        if drop_last:
            self.num_samples = n // self.num_replicas
        else:
            self.num_samples = math.ceil(n / self.num_replicas)
        self.total_size = self.num_samples * self.num_replicas

    def _order(self, cycle: int) -> list[int]:
        if self.shuffle:
            g = torch.Generator().manual_seed(self.seed + cycle)
            order = torch.randperm(self.dataset_size, generator=g).tolist()
        else:
            order = list(range(self.dataset_size))
        if len(order) < self.total_size:
            order = (order * math.ceil(self.total_size / len(order)))[: self.total_size]
        return order[: self.total_size]

    def __iter__(self) -> Iterator[int]:
        cycle = 0
        while True:
            yield from self._order(cycle)[self.rank::self.num_replicas]
            cycle += 1

    def __len__(self) -> int:
        return self.num_samples
