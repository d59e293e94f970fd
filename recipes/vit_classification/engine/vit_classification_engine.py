"""ViT image-classification engine (reference: recipes/vit_classification/engine/vit_classification_engine.py:28-136).

Torch ``DataLoader`` over the recipe dataset with ``InfiniteDistributedSampler``
(train) / ``DistributedSampler`` (eval), the engine's ViT classifier wrapped
by ``parallelize_model`` (native flat FSDP by default, torch FSDP2 / DDP with
``impl: torch``), AdamW + warmup-cosine from ``OptimKit``; logs loss and
top-1 accuracy.  With ``optim.mixed_precision: fp32`` the compute weights
stay fp32.
"""

from __future__ import annotations

import torch
from torch.utils.data import DataLoader, DistributedSampler

from mvp_engine.distributed.parallelize import parallelize_model
from mvp_engine.distributed.utils import is_main_process
from mvp_engine.engine import ENGINE_REGISTRY, Engine, TrainStepContext
from mvp_engine.kit import OptimKit
from mvp_engine.utils.log import logger
from mvp_engine.utils.misc import calculate_model_size

from ..configs.schema import ViTClassificationConfig
from ..dataset import InfiniteDistributedSampler, build_dataset
from ..model import build_vit_model


@ENGINE_REGISTRY.register()
class ViTClassificationEngine(Engine):
    ConfigClass = ViTClassificationConfig
    config: ViTClassificationConfig

    def __init__(self, config):
        super().__init__(config)
        self.optim_kit = OptimKit()

    def prepare_dataloader(self, workflow: str = "train") -> DataLoader:
        dataset = build_dataset(self.config, workflow)
        dp = self.parallel_mesh.dp
        train = workflow == "train"
        if train:
            sampler = InfiniteDistributedSampler(dataset, num_replicas=dp.world_size, rank=dp.rank, shuffle=True,
                                                 seed=int(self.config.seed))
        else:
            sampler = DistributedSampler(dataset, num_replicas=dp.world_size, rank=dp.rank, shuffle=False)
        nw = int(self.config.data.num_workers)
        return DataLoader(dataset, batch_size=int(self.config.data.batch_size), sampler=sampler, num_workers=nw,
                          pin_memory=self.device.type == "cuda", drop_last=train, persistent_workers=nw > 0)

    def _backend_kwargs(self) -> dict:
        kw = self.config.parallel.backend_kwargs.model_dump()
        if str(self.config.optim.mixed_precision) == "fp32":
            fsdp2 = dict(kw.get("fsdp2") or {})
            mp = dict(fsdp2.get("mp_policy") or {})
            mp.update(param_dtype="float32", reduce_dtype="float32", output_dtype="float32")
            fsdp2["mp_policy"] = mp
            kw["fsdp2"] = fsdp2
        return kw

    def prepare_model(self) -> torch.nn.Module:
        native = self.config.parallel.backend_kwargs.impl == "native"
        meta = native and not self.config.model.load_pretrained_weights
        model = build_vit_model(self.config.model, seed=int(self.config.seed), device="meta" if meta else None)
        if not meta:
            model = model.to(self.device)
        logger.info(f" - Model name: {type(model).__name__}")
        wrapped = parallelize_model(model, parallel_mesh=self.parallel_mesh, backend_kwargs=self._backend_kwargs(),
                                    device=self.device)
        if is_main_process():
            total, trainable = calculate_model_size(wrapped)
            logger.info(f" - Model size: {total / 1e9:.4f} B")
            logger.info(f" - Trainable model size: {trainable / 1e9:.4f} B")
        return wrapped

    def prepare_optimizer(self) -> torch.optim.Optimizer:
        return self.optim_kit.build_optimizer(self.model, optimizer="AdamW", lr=float(self.config.optim.lr),
                                              weight_decay=float(self.config.optim.weight_decay))

    def prepare_scheduler(self):
        warmup = int(self.total_steps * float(self.config.optim.warmup_ratio))
        return self.optim_kit.build_lr_scheduler(optimizer=self.optimizer, lr_scheduler="cosine",
                                                 num_warmup_steps=warmup, num_training_steps=self.total_steps)

    def train_pre_step(self, ctx: TrainStepContext) -> TrainStepContext:
        pixel_values, labels = ctx.data
        ctx.data = {"pixel_values": pixel_values.to(self.device, non_blocking=True),
                    "labels": torch.as_tensor(labels).to(self.device, non_blocking=True)}
        return ctx

    def forward_step(self, ctx: TrainStepContext) -> None:
        data = ctx.data
        with torch.autocast(device_type=self.device_type, dtype=self.dtype,
                            enabled=self.dtype != torch.float32 and self.device_type == "cuda"):
            out = self.model(pixel_values=data["pixel_values"], labels=data["labels"])
        acc = (out["logits"].argmax(dim=-1) == data["labels"]).float().mean()
        ctx.outputs = {"loss": out["loss"], "logs": {"train/loss": out["loss"].detach(), "train/acc1": acc.detach()}}

    def train_post_step(self, ctx: TrainStepContext) -> None:
        logs = ctx.outputs["logs"]
        for k in ("train/loss", "train/acc1"):
            if isinstance(logs.get(k), torch.Tensor):
                logs[k] = float(logs[k])
        self.last_logs = dict(logs)
        super().train_post_step(ctx)
