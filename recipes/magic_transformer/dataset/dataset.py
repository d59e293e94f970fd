"""Fake autoregressive data (reference: recipes/magic_transformer/dataset/dataset.py:11-58): sample i is
``seq_len + 1`` uniform token ids drawn from a generator seeded with ``seed + i``; inputs are the first
``seq_len``, labels the last ``seq_len``."""

from __future__ import annotations

import torch
from torch.utils.data import Dataset


class FakeAutoregressiveDataset(Dataset):
    def __init__(self, *, size: int, seq_len: int, vocab_size: int, seed: int) -> None:
        self.size, self.seq_len, self.vocab_size, self.seed = int(size), int(seq_len), int(vocab_size), int(seed)

    def __len__(self) -> int:
        return self.size

    def __getitem__(self, index: int) -> dict[str, torch.Tensor]:
        g = torch.Generator().manual_seed(self.seed + int(index))
        t = torch.randint(0, self.vocab_size, (self.seq_len + 1,), generator=g)
        return {"input_ids": t[:-1].clone(), "labels": t[1:].clone()}


def build_dataset(config, workflow: str = "train") -> FakeAutoregressiveDataset:
    train = workflow == "train"
    d = config.data
    return FakeAutoregressiveDataset(size=d.fake_train_size if train else d.fake_eval_size, seq_len=d.seq_len,
                                     vocab_size=d.vocab_size, seed=int(config.seed) + (0 if train else 10_000))
