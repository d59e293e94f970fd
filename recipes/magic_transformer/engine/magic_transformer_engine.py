"""Magic Transformer engine.

Behaviour of the reference's ``recipes/magic_transformer/engine/magic_transformer_engine.py:28-138``:
fake token data on an endless rank-sharded sampler, the recipe model wrapped by
``parallelize_model`` (DDP with unused-parameter tracking by default), AdamW + warm-up cosine,
mean next-token cross-entropy; logs loss and token accuracy.  The shared plumbing is
:class:`~mvp_engine.engine.map_style.MapStyleEngine`.
"""

from __future__ import annotations

from typing import TypedDict

import torch
import torch.nn.functional as F

from mvp_engine.engine import ENGINE_REGISTRY, TrainStepContext
from mvp_engine.engine.map_style import MapStyleEngine

from ..configs.schema import MagicTransformerConfig
from ..dataset import InfiniteDistributedSampler, build_dataset
from ..model import build_magic_transformer_model


class TrainBatch(TypedDict):
    """A training batch on the device: token ids and next-token labels, both ``[B, T]``."""

    input_ids: torch.Tensor
    labels: torch.Tensor


@ENGINE_REGISTRY.register()
class MagicTransformerEngine(MapStyleEngine):
    ConfigClass = MagicTransformerConfig
    config: MagicTransformerConfig
    sampler_cls = InfiniteDistributedSampler

    def build_dataset(self, workflow: str):
        return build_dataset(self.config, workflow)

    def build_model(self) -> torch.nn.Module:
        return build_magic_transformer_model(self.config.model).to(self.device)

    def train_pre_step(self, ctx: TrainStepContext) -> TrainStepContext:
        ctx.data = self.to_device(input_ids=ctx.data["input_ids"], labels=ctx.data["labels"])
        return ctx

    def forward_step(self, ctx: TrainStepContext) -> None:
        ids, target = ctx.data["input_ids"], ctx.data["labels"]
        mixed = self.dtype != torch.float32
        with torch.autocast(device_type=self.device_type, dtype=self.dtype, enabled=mixed):
            logits = self.model(input_ids=ids)
            loss = F.cross_entropy(logits.flatten(0, -2).float(), target.flatten())
        hits = logits.argmax(-1).eq(target).float().mean()
        ctx.outputs = {"loss": loss, "logs": {"train/loss": float(loss.detach()), "train/token_acc": float(hits)}}
