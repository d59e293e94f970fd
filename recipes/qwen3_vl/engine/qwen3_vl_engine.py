"""Qwen3-VL full-SFT engine (reference: recipes/qwen3_vl/engine/qwen3_vl_engine.py:42-426).

Same loop as the Qwen3 recipe plus the multimodal pieces of the reference:
``MLLMDataKit`` pipeline (Qwen chat schema, image rendering, multi-pack
best-fit packing), step estimation when ``loop.total_steps == -1``, the
Qwen3-VL patches (fp32 patch-embed, VL FLOPs incl. ViT + merger), freeze
flags for ViT / projector / LLM, token-normalised loss and MFU logs.

B200 specifics: the model is built on the meta device and materialised into
the native data-parallel runtime's flat buffers; all per-batch metadata
(3-D M-RoPE positions, document cu_seqlens, vision rotary/interpolation
tables) is built on the host from the pinned CPU batch and copied to the GPU
asynchronously; step time is device time (max over ranks).
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import torch

from mvp_engine.distributed.parallelize import parallelize_model, resolve_impl
from mvp_engine.engine import ENGINE_REGISTRY, Engine, TrainStepContext
from mvp_engine.kit import MFUKit, OptimKit, TokenNormedLossKit
from mvp_engine.kit.mllm import (MLLMDataKit, MLLMDataSpec, MLLMLoaderSpec, MLLMModelKit, MLLMPackingSpec,
                                 MLLMSampleSpec, MLLMSourceSpec, MLLMStepEstimationKit, QwenVLChatSchemaHandler,
                                 QwenVLMediaHandler, QwenVLTokenizationHandler)
from mvp_engine.kit.mllm.data import SyntheticVLSchemaHandler
from mvp_engine.utils.log import logger
from mvp_engine.utils.training import accumulate_gradients, clip_grad_norm_

from ..configs.schema import Qwen3VLConfig
from ..model import patch_qwen3vl_conv3d, patch_qwen3vl_model_flops, prepare_packed_model_inputs


@ENGINE_REGISTRY.register()
class Qwen3VLEngine(Engine):
    ConfigClass = Qwen3VLConfig
    config: Qwen3VLConfig

    def __init__(self, config):
        super().__init__(config)
        if self.parallel_mesh.has_dim("context") and self.parallel_mesh.cp.active:
            # the packed rows carry image features at placeholder positions; cutting them into context
            # chunks would need the vision outputs scattered per chunk, which this recipe does not do
            raise ValueError("the Qwen3-VL recipe does not support context parallelism (parallel.mesh.context)")
        self.config.resolve_batching_config(data_parallel_world_size=self.parallel_mesh.dp.world_size)
        self.data_kit = MLLMDataKit()
        self.model_kit = MLLMModelKit()
        self.step_estimation_kit = MLLMStepEstimationKit()
        self.mfu_kit = MFUKit()
        self.optim_kit = OptimKit()
        self.token_loss_kit = TokenNormedLossKit(device=self.device, dp_world_size=self.parallel_mesh.dp.world_size,
                                                 dp_group=self.parallel_mesh.dp.group)
        o = self.config.optim
        self.token_loss_kit.build_loss_guard(spike_multiplier=o.loss_spike_skip_multiplier,
                                             window_size=int(o.loss_spike_skip_window_size),
                                             min_history=int(o.loss_spike_skip_min_history))

    # --------------------------------------------------------------- data
    def _synthetic(self) -> bool:
        d = self.config.data
        return d.dataset_source.startswith("synthetic") or d.train_path.startswith("synthetic")

    def _data_spec(self, *, resample: bool, resolve_refs: bool) -> MLLMDataSpec:
        d = self.config.data
        if self._synthetic():
            schema = SyntheticVLSchemaHandler()
        else:
            schema = QwenVLChatSchemaHandler(processor=self.processor, thinking_mode=d.thinking_mode)
        sample = MLLMSampleSpec(schema_handler=schema, media_handler=QwenVLMediaHandler(processor=self.processor),
                                tokenization_handler=QwenVLTokenizationHandler(
                                    tokenizer=self.processor.tokenizer, max_seq_len=int(d.max_seq_len)))
        source = "synthetic_mm" if self._synthetic() else d.dataset_source
        return MLLMDataSpec(
            source=MLLMSourceSpec(dataset_path=d.train_path, dataset_source=source, ref_columns=tuple(d.ref_columns),
                                  seed=int(self.config.seed), resample=resample, resolve_refs=resolve_refs),
            sample=sample,
            packing=MLLMPackingSpec(max_seq_len=int(d.max_seq_len), algorithm="multi_pack",
                                    selection_strategy=d.packing_selection_strategy,
                                    open_pack_limit=int(d.packing_open_pack_limit),
                                    buffer_size=int(d.packing_buffer_size), block_causal=True),
            loader=MLLMLoaderSpec(batch_size=int(d.batch_size), num_workers=int(d.num_workers)),
            distribution=self.data_kit.build_distribution_spec(parallel_mesh=self.parallel_mesh),
        )

    def prepare_dataloader(self, workflow: str = "train"):
        if workflow != "train":
            logger.warning(f"Qwen3-VL engine does not support workflow '{workflow}'.")
            return None
        m = self.config.model
        self.processor = self.data_kit.build_processor(
            "synthetic" if self._synthetic() else m.pretrained_model_name_or_path,
            image_max_pixels=m.image_max_pixels)
        if int(self.config.loop.total_steps) == -1:
            est_spec = self._data_spec(resample=False, resolve_refs=False)
            if self._synthetic():
                raise ValueError("`loop.total_steps=-1` needs a finite dataset with a row_count in its meta file")
            meta = json.loads(Path(self.config.data.train_path).read_text())
            est = self.step_estimation_kit.estimate_total_steps(
                self.data_kit.build_dataset(est_spec), total_source_samples=int(meta["row_count"]),
                batch_size=int(self.config.data.batch_size),
                gradient_accumulation_steps=int(self.config.optim.gradient_accumulation_steps),
                data_parallel_world_size=self.parallel_mesh.dp.world_size,
                data_parallel_group=self.parallel_mesh.dp.group, device=self.device)
            self.config.loop.total_steps = est.total_steps
        spec = self._data_spec(resample=True, resolve_refs=True)
        return self.data_kit.build_dataloader(self.data_kit.build_dataset(spec), spec, device=self.device)

    # -------------------------------------------------------------- model
    def _native(self) -> bool:
        return resolve_impl(self.config.parallel.backend_kwargs) == "native"

    def prepare_model(self) -> torch.nn.Module:
        m = self.config.model
        build_device = "meta" if (self._native() and not m.load_pretrained_model) else self.device
        model = self.model_kit.build_model(m.pretrained_model_name_or_path, load_pretrained_model=m.load_pretrained_model,
                                           random_init_seed=int(self.config.seed), device=build_device,
                                           **m.config_overrides)
        logger.info(f"Model name: {type(model).__name__}")
        model = self.model_kit.apply_model_patches(model, [patch_qwen3vl_conv3d, patch_qwen3vl_model_flops])
        model = self.token_loss_kit.apply_chunked_token_loss_patch(model)
        model = self.model_kit.apply_freeze_policy(model, freeze_vit=m.freeze_vit, freeze_projector=m.freeze_projector,
                                                   freeze_llm=m.freeze_llm)
        if build_device != "meta":
            for p in model.parameters():
                if p.requires_grad and p.dtype != torch.float32:
                    p.data = p.data.float()
        if m.gradient_checkpointing.enabled:
            model = self.model_kit.apply_gradient_checkpointing(
                model, use_reentrant=m.gradient_checkpointing.use_reentrant, mode="hf",
                num_layers=m.gradient_checkpointing.num_layers)
        if m.compile.enabled:
            model = self.model_kit.apply_model_compile(model, backend=m.compile.backend, mode=m.compile.mode)
        return parallelize_model(model, parallel_mesh=self.parallel_mesh,
                                 backend_kwargs=self.config.parallel.backend_kwargs.model_dump(), device=self.device)

    def prepare_optimizer(self) -> torch.optim.Optimizer:
        o = self.config.optim
        return self.optim_kit.build_optimizer(self.model, optimizer=o.optimizer, lr=float(o.lr),
                                              weight_decay=float(o.weight_decay))

    def prepare_scheduler(self):
        warmup = math.ceil(self.total_steps * float(self.config.optim.warmup_ratio))
        return self.optim_kit.build_lr_scheduler(optimizer=self.optimizer, lr_scheduler="cosine",
                                                 num_warmup_steps=warmup, num_training_steps=self.total_steps)

    # -------------------------------------------------------------- steps
    _MODEL_KEYS = ("input_ids", "labels", "position_ids", "cu_seq_lens_q", "max_length_q", "pixel_values",
                   "image_grid_thw", "vision_meta")

    def train_pre_step(self, ctx: TrainStepContext) -> TrainStepContext:
        m = self.unwrapped_model
        batch = prepare_packed_model_inputs(dict(ctx.data), model_config=m.config, visual=m.model.visual)
        ctx.data = self.data_kit.to_device(batch, self.device)
        if "image_grid_thw" in batch:  # host copy: only host code (metadata, FLOPs) reads it
            ctx.data["image_grid_thw"] = batch["image_grid_thw"]
        if "vision_meta" in batch:
            meta = batch["vision_meta"]
            ctx.data["vision_meta"] = {k: (v if k == "max_len" else v.to(self.device, non_blocking=True))
                                       for k, v in meta.items()}
        return ctx

    def forward_step(self, ctx: TrainStepContext) -> None:
        data = ctx.data
        with torch.autocast(device_type=self.device_type, dtype=self.dtype,
                            enabled=self.dtype != torch.float32 and self.device_type == "cuda"):
            outputs = self.model(**{k: data[k] for k in self._MODEL_KEYS if k in data})
        m = self.config.model
        self.mfu_kit.accumulate_microbatch(model=self.unwrapped_model, batch_size=int(data["input_ids"].shape[0]),
                                           seq_len=int(data["input_ids"].shape[1]),
                                           attention_token_pairs=data.get("attention_token_pairs"),
                                           image_grid_thw=data.get("image_grid_thw"), is_training=True,
                                           freeze_vit=bool(m.freeze_vit), freeze_projector=bool(m.freeze_projector),
                                           freeze_llm=bool(m.freeze_llm))
        ctx.outputs = {"loss": outputs["loss"], "logs": {"train/loss": 0}}

    def backward_step(self, ctx: TrainStepContext) -> None:
        out = ctx.outputs
        assert out is not None and "loss" in out and "logs" in out
        ctx.should_sync = self.ga_state.advance()
        loss_sum = out["loss"].sum()
        eff, tot = int(ctx.data["effective_tokens"]), int(ctx.data["total_tokens"])
        c = self.config
        divisor = int(c.data.batch_size) * int(c.data.max_seq_len) * int(c.optim.gradient_accumulation_steps)
        if not self.token_loss_kit.guard_loss(loss_sum, eff, step=int(self.step)):
            loss_sum = loss_sum * 0.0
        ctx.loss = self.token_loss_kit.accumulate_microbatch(loss_sum=loss_sum, effective_tokens=eff,
                                                             total_tokens=tot, backward_divisor=divisor)
        with accumulate_gradients(self.model, sync=ctx.should_sync):
            self.scaler.scale(ctx.loss).backward()

    def optimizer_step(self, ctx: TrainStepContext) -> None:
        if not ctx.should_sync:
            return
        stats = self.token_loss_kit.reduce_window()
        self.scaler.unscale_(self.optimizer)
        self.token_loss_kit.rescale_gradients(self.model if hasattr(self.model, "scale_gradients_")
                                              else self.model.parameters(), stats)
        if self.config.optim.clip_grad_norm is not None:
            clip_grad_norm_(self.model, self.config.optim.clip_grad_norm)
        lrs = [float(g["lr"]) for g in self.optimizer.param_groups]
        self.scaler.step(self.optimizer)
        self.scaler.update()
        self.scheduler.step()
        self.optimizer.zero_grad(set_to_none=True)
        out = ctx.outputs
        out["global_total_token_count"] = stats.global_total_tokens
        out["global_effective_token_count"] = stats.global_effective_tokens
        out["global_loss_sum"] = stats.global_loss_sum
        out["step_lrs"] = lrs
        ctx.optimizer_step_completed = True
        self.token_loss_kit.reset()

    def train_post_step(self, ctx: TrainStepContext) -> None:
        out = ctx.outputs
        host_time = float(self.timer.progress_time_latest)
        step_time = self.step_time_ms / 1e3 if self.step_time_ms > 0 else host_time
        tot, eff = int(out["global_total_token_count"]), int(out["global_effective_token_count"])
        logs = out["logs"]
        logs.update({
            "train/loss": float(out["global_loss_sum"] / max(1, eff)),
            "eta": self.timer.eta_string,
            "perf/batch_time": host_time,
            "perf/step_time": step_time,
            "perf/data_time": self.timer.get_scope_time("data_time"),
            "perf/exec_time": self.timer.get_scope_time("exec_time"),
            "perf/toks_per_sec": tot / step_time if step_time > 0 else 1e-8,
            "tokens/total": tot,
            "tokens/effective": eff,
        })
        logs.update(self.mfu_kit.build_log(device_type=self.device.type,
                                           precision=str(self.config.optim.mixed_precision),
                                           step_time_seconds=step_time))
        for i, lr in enumerate(out["step_lrs"]):
            logs[f"lr/group_{i}"] = lr
        self.last_logs = dict(logs)
        logger.log_metrics(logs, step=self.step, total_steps=self.total_steps)
