"""Magic Transformer engine (reference: recipes/magic_transformer/engine/magic_transformer_engine.py:28-138):
fake token data with a never-ending rank-sharded sampler, the recipe model wrapped by
``parallelize_model`` (DDP with unused-parameter tracking by default), AdamW + warmup-cosine,
mean next-token cross-entropy; logs loss and token accuracy."""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch.utils.data import DataLoader, DistributedSampler

from mvp_engine.distributed.parallelize import parallelize_model
from mvp_engine.engine import ENGINE_REGISTRY, Engine, TrainStepContext
from mvp_engine.kit import OptimKit
from mvp_engine.utils.log import logger

from ..configs.schema import MagicTransformerConfig
from ..dataset import InfiniteDistributedSampler, build_dataset
from ..model import build_magic_transformer_model


@ENGINE_REGISTRY.register()
class MagicTransformerEngine(Engine):
    ConfigClass = MagicTransformerConfig
    config: MagicTransformerConfig

    def __init__(self, config):
        super().__init__(config)
        self.optim_kit = OptimKit()

    def prepare_dataloader(self, workflow: str = "train") -> DataLoader:
        ds = build_dataset(self.config, workflow)
        dp = self.parallel_mesh.dp
        train = workflow == "train"
        sampler = (InfiniteDistributedSampler(ds, num_replicas=dp.world_size, rank=dp.rank, shuffle=True,
                                              seed=int(self.config.seed)) if train
                   else DistributedSampler(ds, num_replicas=dp.world_size, rank=dp.rank, shuffle=False))
        nw = int(self.config.data.num_workers)
        return DataLoader(ds, batch_size=int(self.config.data.batch_size), sampler=sampler, num_workers=nw,
                          pin_memory=self.device.type == "cuda", drop_last=train, persistent_workers=nw > 0)

    def prepare_model(self) -> torch.nn.Module:
        model = build_magic_transformer_model(self.config.model).to(self.device)
        logger.info(f" - Model name: {type(model).__name__}")
        return parallelize_model(model, parallel_mesh=self.parallel_mesh,
                                 backend_kwargs=self.config.parallel.backend_kwargs.model_dump(), device=self.device)

    def prepare_optimizer(self) -> torch.optim.Optimizer:
        return self.optim_kit.build_optimizer(self.model, optimizer="AdamW", lr=float(self.config.optim.lr),
                                              weight_decay=float(self.config.optim.weight_decay))

    def prepare_scheduler(self):
        warmup = int(self.total_steps * float(self.config.optim.warmup_ratio))
        return self.optim_kit.build_lr_scheduler(optimizer=self.optimizer, lr_scheduler="cosine",
                                                 num_warmup_steps=warmup, num_training_steps=self.total_steps)

    def train_pre_step(self, ctx: TrainStepContext) -> TrainStepContext:
        ctx.data = {k: ctx.data[k].to(self.device, non_blocking=True) for k in ("input_ids", "labels")}
        return ctx

    def forward_step(self, ctx: TrainStepContext) -> None:
        d = ctx.data
        with torch.autocast(device_type=self.device_type, dtype=self.dtype, enabled=self.dtype != torch.float32):
            logits = self.model(input_ids=d["input_ids"])
            loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), d["labels"].reshape(-1))
        acc = (logits.argmax(-1) == d["labels"]).float().mean()
        ctx.outputs = {"loss": loss, "logs": {"train/loss": float(loss.detach()), "train/token_acc": float(acc)}}
