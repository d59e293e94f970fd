"""ViT image-classification engine.

Behaviour of the reference's ``recipes/vit_classification/engine/vit_classification_engine.py:28-136``:
the recipe dataset on an endless rank-sharded sampler (evaluation: ``DistributedSampler``), the
ViT classifier wrapped by ``parallelize_model`` (native flat FSDP by default, torch FSDP2 / DDP
with ``impl: torch``), AdamW + warm-up cosine; logs loss and top-1 accuracy.  With
``optim.mixed_precision: fp32`` the FSDP2 mixed-precision policy is forced to fp32 so the
compute weights stay fp32.  The shared plumbing is :class:`~mvp_engine.engine.map_style.MapStyleEngine`.
"""

from __future__ import annotations

from typing import TypedDict

import torch

from mvp_engine.distributed.parallelize import resolve_impl
from mvp_engine.distributed.utils import is_main_process
from mvp_engine.engine import ENGINE_REGISTRY, TrainStepContext
from mvp_engine.engine.map_style import MapStyleEngine
from mvp_engine.utils.log import logger
from mvp_engine.utils.misc import calculate_model_size

from ..configs.schema import ViTClassificationConfig
from ..dataset import InfiniteDistributedSampler, build_dataset
from ..model import build_vit_model

_FP32_POLICY = {"param_dtype": "float32", "reduce_dtype": "float32", "output_dtype": "float32"}


class TrainBatch(TypedDict):
    """A training batch on the device: images ``[B, 3, H, W]`` and class labels ``[B]``."""

    pixel_values: torch.Tensor
    labels: torch.Tensor


@ENGINE_REGISTRY.register()
class ViTClassificationEngine(MapStyleEngine):
    ConfigClass = ViTClassificationConfig
    config: ViTClassificationConfig
    sampler_cls = InfiniteDistributedSampler

    def build_dataset(self, workflow: str):
        return build_dataset(self.config, workflow)

    def parallel_backend_kwargs(self) -> dict:
        kw = super().parallel_backend_kwargs()
        if str(self.config.optim.mixed_precision) == "fp32":
            fsdp2 = dict(kw.get("fsdp2") or {})
            fsdp2["mp_policy"] = {**(fsdp2.get("mp_policy") or {}), **_FP32_POLICY}
            kw["fsdp2"] = fsdp2
        return kw

    def build_model(self) -> torch.nn.Module:
        on_meta = resolve_impl(self.config.parallel.backend_kwargs) == "native" and not self.config.model.load_pretrained_weights
        model = build_vit_model(self.config.model, seed=int(self.config.seed), device="meta" if on_meta else None)
        return model if on_meta else model.to(self.device)

    def prepare_model(self) -> torch.nn.Module:
        wrapped = super().prepare_model()
        if is_main_process():
            total, trainable = calculate_model_size(wrapped)
            logger.info(f" - Model size: {total / 1e9:.4f} B")
            logger.info(f" - Trainable model size: {trainable / 1e9:.4f} B")
        return wrapped

    def train_pre_step(self, ctx: TrainStepContext) -> TrainStepContext:
        pixels, classes = ctx.data
        ctx.data = self.to_device(pixel_values=pixels, labels=classes)
        return ctx

    def forward_step(self, ctx: TrainStepContext) -> None:
        batch = ctx.data
        autocast = self.dtype != torch.float32 and self.device_type == "cuda"
        with torch.autocast(device_type=self.device_type, dtype=self.dtype, enabled=autocast):
            out = self.model(pixel_values=batch["pixel_values"], labels=batch["labels"])
        top1 = out["logits"].argmax(dim=-1).eq(batch["labels"]).float().mean()
        ctx.outputs = {"loss": out["loss"], "logs": {"train/loss": out["loss"].detach(), "train/acc1": top1.detach()}}

    def train_post_step(self, ctx: TrainStepContext) -> None:
        logs = ctx.outputs["logs"]
        logs.update({k: float(v) for k, v in logs.items() if isinstance(v, torch.Tensor)})
        super().train_post_step(ctx)
