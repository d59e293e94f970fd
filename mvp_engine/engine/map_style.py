"""Engine base for recipes that train on a map-style dataset with AdamW + warmup-cosine.

The ViT-classification and MagicTransformer recipes (reference: their ``engine/*_engine.py``)
share everything around the model: an endless rank-sharded sampler for training, a plain
``DistributedSampler`` for evaluation, AdamW from ``OptimKit`` and a cosine schedule whose
warm-up is ``optim.warmup_ratio`` of the run.  They differ only in the dataset, the model and
the step; :class:`MapStyleEngine` holds the shared part and asks subclasses for the rest
through :meth:`build_dataset`, :meth:`build_model` and the usual step hooks.
"""

from __future__ import annotations

from typing import Any

import torch
from torch.utils.data import DataLoader, DistributedSampler

from ..distributed.parallelize import parallelize_model
from ..utils.log import logger
from .engine import Engine


class MapStyleEngine(Engine):
    """``prepare_dataloader`` / ``prepare_model`` / ``prepare_optimizer`` / ``prepare_scheduler`` from config."""

    sampler_cls: Any = None  # endless rank-sharded sampler class (set by the recipe)

    def __init__(self, config):
        super().__init__(config)
        from ..kit import OptimKit

        self.optim_kit = OptimKit()

    # ---- recipe hooks
    def build_dataset(self, workflow: str):
        raise NotImplementedError

    def build_model(self) -> torch.nn.Module:
        raise NotImplementedError

    def parallel_backend_kwargs(self) -> dict:
        return self.config.parallel.backend_kwargs.model_dump()

    # ---- shared plumbing
    def _sampler(self, dataset, training: bool):
        dp = self.parallel_mesh.dp
        if training:
            return self.sampler_cls(dataset, num_replicas=dp.world_size, rank=dp.rank, shuffle=True,
                                    seed=int(self.config.seed))
        return DistributedSampler(dataset, num_replicas=dp.world_size, rank=dp.rank, shuffle=False)

    def prepare_dataloader(self, workflow: str = "train") -> DataLoader:
        training = workflow == "train"
        dataset = self.build_dataset(workflow)
        workers = int(self.config.data.num_workers)
        return DataLoader(dataset, batch_size=int(self.config.data.batch_size),
                          sampler=self._sampler(dataset, training), num_workers=workers,
                          pin_memory=self.device.type == "cuda", drop_last=training, persistent_workers=workers > 0)

    def prepare_model(self) -> torch.nn.Module:
        model = self.build_model()
        logger.info(f" - Model name: {type(model).__name__}")
        return parallelize_model(model, parallel_mesh=self.parallel_mesh, backend_kwargs=self.parallel_backend_kwargs(),
                                 device=self.device)

    def prepare_optimizer(self) -> torch.optim.Optimizer:
        o = self.config.optim
        return self.optim_kit.build_optimizer(self.model, optimizer="AdamW", lr=float(o.lr),
                                              weight_decay=float(o.weight_decay))

    def prepare_scheduler(self):
        steps = self.total_steps
        return self.optim_kit.build_lr_scheduler(optimizer=self.optimizer, lr_scheduler="cosine",
                                                 num_warmup_steps=int(steps * float(self.config.optim.warmup_ratio)),
                                                 num_training_steps=steps)

    def to_device(self, **tensors: Any) -> dict[str, torch.Tensor]:
        return {k: torch.as_tensor(v).to(self.device, non_blocking=True) for k, v in tensors.items()}
