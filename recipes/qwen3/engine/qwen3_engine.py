"""Qwen3 text pretraining engine (reference: recipes/qwen3/engine/qwen3_engine.py:36-368).

Same structure as the reference recipe: LLMDataKit packing pipeline, model
kit (build -> FLOPs patch -> token-loss patch -> freeze -> checkpointing ->
parallelize), AdamW + cosine schedule, token-normalised loss with the
per-window gradient rescale, global-norm clip, MFU / tokens-per-second logs.

B200 specifics: the model is built on the meta device and materialised
straight into the native data-parallel runtime's flat buffers; the
token-normalisation scale and the clip coefficient are folded into the fused
optimizer update; step time is the device time of the step (max over ranks).
"""

from __future__ import annotations

import math
from typing import Any

import torch

from mvp_engine.distributed.parallelize import parallelize_model, resolve_impl
from mvp_engine.engine import ENGINE_REGISTRY, Engine, TrainStepContext
from mvp_engine.kit import (LLMDataKit, LLMDataSpec, LLMLoaderSpec, LLMModelKit, LLMPackingSpec,
                            LLMPretrainTextSchemaHandler, LLMPretrainTextTokenizationHandler, LLMSampleSpec,
                            LLMSourceSpec, LLMStepEstimationKit, LLMTokenIdsSchemaHandler, MFUKit, OptimKit,
                            TokenNormedLossKit)
from mvp_engine.kit.llm import ModelInputs
from mvp_engine.parallel.context import maybe_shard_batch
from mvp_engine.utils.log import logger
from mvp_engine.utils.training import accumulate_gradients, clip_grad_norm_

from ..configs.schema import Qwen3Config
from ..model import patch_qwen3_model_flops, prepare_packed_model_inputs


@ENGINE_REGISTRY.register()
class Qwen3Engine(Engine):
    ConfigClass = Qwen3Config
    config: Qwen3Config

    def __init__(self, config):
        super().__init__(config)
        self.config.resolve_batching_config(data_parallel_world_size=self.parallel_mesh.dp.world_size)
        self.data_kit = LLMDataKit()
        self.model_kit = LLMModelKit()
        self.step_estimation_kit = LLMStepEstimationKit()
        self.mfu_kit = MFUKit()
        self.optim_kit = OptimKit()
        # token counts / loss sums reduce over every rank that holds part of a step's tokens
        # (data x context parallel ranks)
        red = self.parallel_mesh.dp_cp
        tp = self.parallel_mesh.tp
        sp = tp.active and bool(self.config.parallel.backend_kwargs.sequence_parallel)
        self.token_loss_kit = TokenNormedLossKit(device=self.device, dp_world_size=red.world_size, dp_group=red.group,
                                                 loss_sum_group=tp.group if sp else None)
        o = self.config.optim
        self.token_loss_kit.build_loss_guard(spike_multiplier=o.loss_spike_skip_multiplier,
                                             window_size=int(o.loss_spike_skip_window_size),
                                             min_history=int(o.loss_spike_skip_min_history))

    # --------------------------------------------------------------- data
    def _data_spec(self, *, resample: bool, shuffle: str, drop_last: bool = True) -> LLMDataSpec:
        d = self.config.data
        synthetic = d.dataset_source.startswith("synthetic") or d.train_path.startswith("synthetic")
        schema = LLMTokenIdsSchemaHandler() if synthetic else LLMPretrainTextSchemaHandler(text_field=d.text_field)
        sample = LLMSampleSpec(schema_handler=schema,
                               tokenization_handler=LLMPretrainTextTokenizationHandler(
                                   tokenizer=self.tokenizer, max_seq_len=int(d.max_seq_len),
                                   add_eos=not synthetic))
        source = "synthetic_text" if synthetic and not d.dataset_source.startswith("synthetic") else d.dataset_source
        return LLMDataSpec(
            source=LLMSourceSpec(dataset_path=d.train_path, dataset_source=source, seed=int(self.config.seed),
                                 resample=resample, shuffle_mode=shuffle),
            sample=sample,
            packing=LLMPackingSpec(max_seq_len=int(d.max_seq_len), tail_policy=d.packing_tail_policy,
                                   isolate_attention=d.packing_isolate_attention,
                                   isolate_position_ids=d.packing_isolate_position_ids),
            loader=LLMLoaderSpec(batch_size=int(d.batch_size), num_workers=int(d.num_workers), drop_last=drop_last),
            distribution=self.data_kit.build_distribution_spec(parallel_mesh=self.parallel_mesh),
        )

    def prepare_dataloader(self, workflow: str = "train"):
        if workflow != "train":
            logger.warning(f"Qwen3 pretrain engine does not support workflow '{workflow}'.")
            return None
        d = self.config.data
        synthetic = d.dataset_source.startswith("synthetic") or d.train_path.startswith("synthetic")
        self.tokenizer = self.data_kit.build_tokenizer(
            "synthetic" if synthetic else self.config.model.pretrained_model_name_or_path)
        if int(self.config.loop.total_steps) == -1:
            est = self.step_estimation_kit.estimate_total_steps(
                self.data_kit.build_dataset(self._data_spec(resample=False, shuffle="none", drop_last=False)),
                batch_size=int(d.batch_size), gradient_accumulation_steps=int(self.config.optim.gradient_accumulation_steps),
                data_parallel_world_size=self.parallel_mesh.dp.world_size,
                data_parallel_group=self.parallel_mesh.dp.group, device=self.device)
            self.config.loop.total_steps = est.total_steps
        spec = self._data_spec(resample=True, shuffle="chunk")
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
        model = self.model_kit.apply_model_patches(model, [patch_qwen3_model_flops])
        model = self.token_loss_kit.apply_chunked_token_loss_patch(model)
        model = self.model_kit.apply_freeze_policy(model, freeze_llm=m.freeze_llm)
        if build_device != "meta":
            for p in model.parameters():
                if p.requires_grad and p.dtype != torch.float32:
                    p.data = p.data.float()
        if m.gradient_checkpointing.enabled:
            model = self.model_kit.apply_gradient_checkpointing(model, use_reentrant=m.gradient_checkpointing.use_reentrant,
                                                                mode="hf", num_layers=m.gradient_checkpointing.num_layers)
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
    def train_pre_step(self, ctx: TrainStepContext) -> TrainStepContext:
        batch = maybe_shard_batch(self.unwrapped_model, ctx.data)  # context parallel: this rank's chunks (host)
        batch: ModelInputs = self.data_kit.to_device(batch, self.device)
        ctx.data = prepare_packed_model_inputs(batch)
        return ctx

    _MODEL_KEYS = ("input_ids", "labels", "shift_labels", "position_ids", "cu_seq_lens_q", "max_length_q")

    def _loss_grad_hint(self):
        """The per-token gradient the loss will receive, when it is fixed in advance: the token loss is
        backpropagated as ``sum / divisor`` and nothing can change that factor (no loss-spike guard, no fp16
        loss scaling).  The model's LM head then runs its backward in the forward (one logits GEMM, not two)."""
        d = self.config
        if d.optim.loss_spike_skip_multiplier is not None or self.dtype == torch.float16:
            return None
        divisor = int(d.data.batch_size) * int(d.data.max_seq_len) * int(d.optim.gradient_accumulation_steps)
        return float(torch.tensor(1.0, dtype=torch.float32) / divisor)  # the fp32 value autograd will pass

    def forward_step(self, ctx: TrainStepContext) -> None:
        data = ctx.data
        model = self.unwrapped_model
        if hasattr(model, "loss_chunk_size"):
            model.loss_grad_hint = self._loss_grad_hint()
        with torch.autocast(device_type=self.device_type, dtype=self.dtype,
                            enabled=self.dtype != torch.float32 and self.device_type == "cuda"):
            outputs = self.model(**{k: data[k] for k in self._MODEL_KEYS if k in data})
        cp_len = data.get("cp_total_tokens")
        flops = self.unwrapped_model.calculate_model_flops(
            batch_size=int(data["input_ids"].shape[0]), seq_len=int(cp_len or data["input_ids"].shape[1]),
            attention_token_pairs=data.get("attention_token_pairs"), is_training=True,
            freeze_llm=bool(self.config.model.freeze_llm))
        if cp_len:  # each context rank does 1/cp of the row's work
            flops /= self.parallel_mesh.cp.world_size
        flops /= self.parallel_mesh.tp.world_size  # and each tensor rank 1/tp
        self.mfu_kit.accumulate_microbatch(model_flops=flops)
        ctx.outputs = {"loss": outputs["loss"], "logs": {"train/loss": 0}}

    def backward_step(self, ctx: TrainStepContext) -> None:
        out = ctx.outputs
        assert out is not None and "loss" in out and "logs" in out
        ctx.should_sync = self.ga_state.advance()
        loss_sum = out["loss"].sum()
        eff, tot = int(ctx.data["effective_tokens"]), int(ctx.data["total_tokens"])
        d = self.config
        divisor = int(d.data.batch_size) * int(d.data.max_seq_len) * int(d.optim.gradient_accumulation_steps)
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
