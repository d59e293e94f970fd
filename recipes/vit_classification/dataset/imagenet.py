"""Image datasets for ViT classification (reference: recipes/vit_classification/dataset/imagenet.py:14-73).

* ``fake``: torchvision ``FakeData`` through the ImageNet train / eval
  transforms (random-resized crop + flip, or resize + center crop; then
  normalise) — the reference's ``use_fake_data``.
* ``imagefolder``: torchvision ``ImageFolder`` with the same transforms.
* ``gaussian``: pixels ~ N(0, 1) of shape [3, S, S] and labels uniform in
  [0, num_classes), generated from ``(seed, index)`` alone, so a sample is
  the same tensor whichever rank or process draws it.
"""

from __future__ import annotations

from pathlib import Path

import torch
from torch.utils.data import Dataset

IMAGENET_DEFAULT_MEAN: list[float] = [0.485, 0.456, 0.406]
IMAGENET_DEFAULT_STD: list[float] = [0.229, 0.224, 0.225]


def build_transforms(image_size: int, is_train: bool, mean: list[float] | None = None,
                     std: list[float] | None = None):
    from torchvision import transforms

    mean = mean or IMAGENET_DEFAULT_MEAN
    std = std or IMAGENET_DEFAULT_STD
    if is_train:
        ops = [transforms.RandomResizedCrop(image_size), transforms.RandomHorizontalFlip()]
    else:
        ops = [transforms.Resize(int(image_size / 0.875)), transforms.CenterCrop(image_size)]
    return transforms.Compose(ops + [transforms.ToTensor(), transforms.Normalize(mean=mean, std=std)])


class GaussianImageDataset(Dataset):
    def __init__(self, size: int, image_size: int, num_classes: int, seed: int = 0, channels: int = 3) -> None:
        self.size, self.image_size, self.num_classes = int(size), int(image_size), int(num_classes)
        self.seed, self.channels = int(seed), int(channels)

    def __len__(self) -> int:
        return self.size

    def __getitem__(self, index: int):
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + int(index))
        x = torch.randn(self.channels, self.image_size, self.image_size, generator=g)
        y = int(torch.randint(0, self.num_classes, (1,), generator=g))
        return x, y


def build_dataset(config, workflow: str):
    d = config.data
    is_train = workflow == "train"
    source = d.resolved_source()
    size = int(d.fake_train_size if is_train else d.fake_val_size)
    if source == "gaussian":
        return GaussianImageDataset(size, int(d.image_size), int(d.num_classes),
                                    seed=int(getattr(config, "seed", 0)) + (0 if is_train else 1))
    tf = build_transforms(int(d.image_size), is_train, list(d.mean), list(d.std))
    if source == "fake":
        from torchvision import datasets

        return datasets.FakeData(size=size, image_size=(3, int(d.image_size), int(d.image_size)),
                                 num_classes=int(d.num_classes), transform=tf)
    root = Path(d.train_path if is_train else d.val_path)
    if not root.exists():
        raise FileNotFoundError(f"{workflow} dataset path does not exist: {root}. Set data.use_fake_data=true "
                                "for a smoke run, or point train_path/val_path to ImageNet folders.")
    from torchvision import datasets

    return datasets.ImageFolder(root=str(root), transform=tf)
