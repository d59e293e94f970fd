"""Multimodal data kit (reference: mvp_engine/kit/mllm/data/data.py:23-217)."""

from __future__ import annotations

from functools import partial
from operator import methodcaller
from typing import Any

import torch

from ....data import Dataset, RuntimeContext, TorchLoader
from .collator import MLLMBatchCollator
from .guard import MLLMModelInputGuard, MLLMRawRowGuard, MLLMSampleGuard
from .packing import MLLMPackingAssembler
from .qwen.processor import QwenVLImageProcessor, QwenVLProcessor
from .sample import MLLMSample
from .spec import MLLMDataSpec, MLLMDistributionSpec
from .types import ModelInputs


class _SampleAssembler:
    def __init__(self, sample_spec, assemble_context: Any = None) -> None:
        self.sample_spec = sample_spec

    def push(self, row):
        return [MLLMSample.from_row(row, sample_spec=self.sample_spec)]

    def finish(self, *, drop_last: bool = False):
        return []

    def state_dict(self):
        return {}

    def fingerprint(self):
        return type(self).__name__


class MLLMDataKit:
    def build_distribution_spec(self, *, parallel_mesh) -> MLLMDistributionSpec:
        return MLLMDistributionSpec(device_mesh=parallel_mesh.device_mesh, dp_dims=parallel_mesh.dp.dim_names or None)

    def build_processor(self, pretrained_model_name_or_path: str, *, image_min_pixels: int | None = None,
                        image_max_pixels: int | None = None, trust_remote_code: bool = True, **kwargs: Any) -> Any:
        """HF AutoProcessor when available locally; otherwise the built-in Qwen-VL processor."""
        proc = None
        if not pretrained_model_name_or_path.startswith("synthetic"):
            try:
                from transformers import AutoProcessor

                proc = AutoProcessor.from_pretrained(pretrained_model_name_or_path, trust_remote_code=trust_remote_code,
                                                     **kwargs)
            except Exception:
                proc = None
        if proc is None:
            ip = QwenVLImageProcessor(min_pixels=image_min_pixels or 64 * 32 * 32,
                                      max_pixels=image_max_pixels or 1024 * 1024)
            return QwenVLProcessor(image_processor=ip)
        size = dict(getattr(proc.image_processor, "size", {}) or {})
        if image_min_pixels is not None:
            size["shortest_edge"] = int(image_min_pixels)
        if image_max_pixels is not None:
            size["longest_edge"] = int(image_max_pixels)
        proc.image_processor.size = size
        tok = proc.tokenizer
        if tok.pad_token_id is None and tok.eos_token is not None:
            tok.pad_token = tok.eos_token
        return proc

    def build_dataset(self, spec: MLLMDataSpec) -> Dataset:
        src, dspec = spec.source, spec.distribution
        if dspec is None or dspec.device_mesh is None or dspec.dp_dims is None:
            ctx = RuntimeContext.from_runtime(seed=src.seed)
        else:
            ctx = RuntimeContext.from_runtime(seed=src.seed, device_mesh=dspec.device_mesh, dp_dims=dspec.dp_dims)
        ds = Dataset.from_source(src.dataset_source, src.dataset_path, context=ctx, resample=src.resample,
                                 shuffle_mode="chunk" if src.resample else "none")
        ds = ds.assemble(partial(MLLMRawRowGuard, schema_handler=spec.sample.schema_handler))
        ds = ds.assemble(partial(_SampleAssembler, spec.sample))
        ds = ds.assemble(MLLMSampleGuard)
        ds = ds.assemble(partial(spec.packing.assembler_cls or MLLMPackingAssembler, spec.packing))
        ds = ds.map(methodcaller("to_model_inputs"))
        proc = spec.sample.media_handler.processor
        tok = getattr(proc, "tokenizer", proc)
        image_id = tok.convert_tokens_to_ids("<|image_pad|>") if hasattr(tok, "convert_tokens_to_ids") else None
        merge = getattr(getattr(proc, "image_processor", None), "merge_size", 2)
        ds = ds.assemble(partial(MLLMModelInputGuard, ignore_index=spec.sample.tokenization_handler.ignore_index,
                                 image_token_id=image_id, merge_size=merge, verbose=False))
        return ds

    def build_collator(self, spec: MLLMDataSpec) -> MLLMBatchCollator:
        proc = spec.sample.media_handler.processor
        tok = getattr(proc, "tokenizer", proc)
        pad = getattr(tok, "pad_token_id", None)
        if pad is None:
            raise ValueError("Tokenizer must expose a pad_token_id to build an MLLM collator.")
        return MLLMBatchCollator(pad_token_id=int(pad), media_handler=spec.sample.media_handler,
                                 ignore_index=spec.sample.tokenization_handler.ignore_index)

    def build_dataloader(self, dataset: Dataset, spec: MLLMDataSpec, *, device: torch.device | None = None,
                         collate_fn=None):
        ld = spec.loader
        pin = ld.pin_memory if ld.pin_memory is not None else (device is not None and device.type == "cuda")
        return TorchLoader(dataset, num_workers=ld.num_workers, pin_memory=pin, persistent_workers=ld.persistent_workers,
                           multiprocessing_context=ld.multiprocessing_context).batch(
            batch_size=ld.batch_size, drop_last=ld.drop_last, collate_fn=collate_fn or self.build_collator(spec))

    def to_device(self, batch: ModelInputs, device: torch.device) -> ModelInputs:
        out = {}
        for k, v in batch.items():
            if isinstance(v, torch.Tensor):
                out[k] = v.to(device, non_blocking=True)
            elif isinstance(v, dict):
                out[k] = v  # host-side metadata (e.g. vision_meta) is moved where it is used
            else:
                out[k] = v
        return out
