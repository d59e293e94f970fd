"""Minimal VLM engine (reference: recipes/minimal_vlm/engine/minimal_vlm_engine.py:24-158).

No kits beyond data plumbing: padded batches, the model's mean token loss as a scalar, the base
engine's backward / optimizer step, AdamW over trainable parameters with warmup-cosine.  Per batch
the host builds document ``cu_seqlens`` (each row's valid tokens are one document, padding its
own), 3-D M-RoPE positions and the vision metadata.
"""

from __future__ import annotations

import math

import torch

from mvp_engine.data import TorchLoader
from mvp_engine.distributed.parallelize import parallelize_model, resolve_impl
from mvp_engine.engine import ENGINE_REGISTRY, Engine, TrainStepContext
from mvp_engine.kit import OptimKit
from mvp_engine.kit.llm.data.collator import varlen_metadata
from mvp_engine.utils.log import logger
from recipes.qwen3_vl.model.packing import build_qwen3_vl_packed_position_ids

from ..configs.schema import MinimalVLMConfig
from ..dataset import MinimalVLMCollator, build_dataset, build_qwen3_vl_processor
from ..model import build_qwen3_vl_model


@ENGINE_REGISTRY.register()
class MinimalVLMEngine(Engine):
    ConfigClass = MinimalVLMConfig
    config: MinimalVLMConfig
    processor = None

    def prepare_dataloader(self, workflow: str = "train"):
        if workflow != "train":
            logger.warning(f"Minimal VLM engine does not support workflow '{workflow}'.")
            return None
        d = self.config.data
        synthetic = d.dataset_source.startswith("synthetic") or str(d.train_path).startswith("synthetic")
        if self.processor is None:
            self.processor = build_qwen3_vl_processor(self.config.model, synthetic=synthetic)
        dataset = build_dataset(self.config, processor=self.processor, parallel_mesh=self.parallel_mesh)
        loader = TorchLoader(dataset, num_workers=int(d.num_workers), pin_memory=self.device.type == "cuda")
        return loader.batch(batch_size=int(d.batch_size), drop_last=True,
                            collate_fn=MinimalVLMCollator(pad_token_id=int(self.processor.tokenizer.pad_token_id)))

    def prepare_model(self) -> torch.nn.Module:
        native = resolve_impl(self.config.parallel.backend_kwargs) == "native"
        meta = native and not self.config.model.load_pretrained_model
        model = build_qwen3_vl_model(self.config.model, seed=int(self.config.seed),
                                     device="meta" if meta else self.device)
        logger.info(f"Model name: {type(model).__name__}")
        return parallelize_model(model, parallel_mesh=self.parallel_mesh,
                                 backend_kwargs=self.config.parallel.backend_kwargs.model_dump(), device=self.device)

    def prepare_optimizer(self) -> torch.optim.Optimizer:
        return OptimKit().build_optimizer(self.model, optimizer="AdamW", lr=float(self.config.optim.lr),
                                          weight_decay=float(self.config.optim.weight_decay))

    def prepare_scheduler(self):
        warmup = math.ceil(self.total_steps * float(self.config.optim.warmup_ratio))
        return OptimKit().build_lr_scheduler(optimizer=self.optimizer, lr_scheduler="cosine",
                                             num_warmup_steps=warmup, num_training_steps=self.total_steps)

    def train_pre_step(self, ctx: TrainStepContext) -> TrainStepContext:
        data = dict(ctx.data)
        m = self.unwrapped_model
        am = data["attention_mask"]
        cu, mx, _ = varlen_metadata(am)  # valid tokens of a row = one document; padding another
        data["position_ids"] = build_qwen3_vl_packed_position_ids(
            input_ids=data["input_ids"], pack_segment_ids=am, image_grid_thw=data.get("image_grid_thw"),
            model_config=m.config)
        data["cu_seq_lens_q"], data["max_length_q"] = cu, mx
        grid = data.get("image_grid_thw")
        meta = m.model.visual.vision_metadata(grid) if grid is not None and grid.numel() else None
        batch = {k: (v.to(self.device, non_blocking=True) if isinstance(v, torch.Tensor) and k != "image_grid_thw"
                     else v) for k, v in data.items()}
        if meta is not None:
            batch["vision_meta"] = {k: (v if k == "max_len" else v.to(self.device, non_blocking=True))
                                    for k, v in meta.items()}
        ctx.data = batch
        return ctx

    def forward_step(self, ctx: TrainStepContext) -> None:
        data = ctx.data
        keys = ("input_ids", "labels", "position_ids", "cu_seq_lens_q", "max_length_q", "pixel_values",
                "image_grid_thw", "vision_meta")
        with torch.autocast(device_type=self.device_type, dtype=self.dtype,
                            enabled=self.dtype != torch.float32 and self.device_type == "cuda"):
            out = self.model(**{k: data[k] for k in keys if k in data})
        n = (torch.nn.functional.pad(data["labels"], (0, 1), value=-100)[..., 1:] != -100).sum().clamp(min=1)
        loss = out["loss"].sum() / n  # the HF causal-LM mean token loss
        ctx.outputs = {"loss": loss, "logs": {"train/loss": float(loss.detach())}}
