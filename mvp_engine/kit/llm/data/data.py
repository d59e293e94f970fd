"""Text-LM data kit (reference: mvp_engine/kit/llm/data/data.py:25-140)."""

from __future__ import annotations

from functools import partial
from operator import methodcaller
from typing import Any

import torch

from ....data import Dataset, RuntimeContext, SyntheticTokenizer, TorchLoader
from .collator import LLMBatchCollator
from .guard import LLMModelInputGuard, LLMRawRowGuard, LLMSampleGuard
from .packing import LLMPackingAssembler
from .sample import LLMSampleAssembler
from .spec import LLMDataSpec, LLMDistributionSpec
from .types import ModelInputs

IGNORE_INDEX = -100


class LLMDataKit:
    def build_distribution_spec(self, *, parallel_mesh) -> LLMDistributionSpec:
        return LLMDistributionSpec(device_mesh=parallel_mesh.device_mesh, dp_dims=parallel_mesh.dp.dim_names or None)

    def build_tokenizer(self, pretrained_model_name_or_path: str, *, trust_remote_code: bool = True,
                        padding_side: str = "right", pad_token_fallback_to_eos: bool = True, **kwargs: Any) -> Any:
        """HF tokenizer when its files are available; otherwise the synthetic stand-in."""
        if pretrained_model_name_or_path.startswith("synthetic"):
            return SyntheticTokenizer()
        try:
            from transformers import AutoTokenizer

            tok = AutoTokenizer.from_pretrained(pretrained_model_name_or_path, trust_remote_code=trust_remote_code,
                                                **kwargs)
        except Exception:
            return SyntheticTokenizer()
        tok.padding_side = padding_side
        if pad_token_fallback_to_eos and tok.pad_token_id is None and tok.eos_token is not None:
            tok.pad_token = tok.eos_token
        return tok

    def build_dataset(self, spec: LLMDataSpec) -> Dataset:
        src, dist_spec = spec.source, spec.distribution
        if dist_spec is None or dist_spec.device_mesh is None or dist_spec.dp_dims is None:
            ctx = RuntimeContext.from_runtime(seed=src.seed)
        else:
            ctx = RuntimeContext.from_runtime(seed=src.seed, device_mesh=dist_spec.device_mesh,
                                              dp_dims=dist_spec.dp_dims)
        ds = Dataset.from_source(src.dataset_source, src.dataset_path, context=ctx, resample=src.resample,
                                 shuffle_mode=src.shuffle_mode)
        ds = ds.assemble(partial(LLMRawRowGuard, schema_handler=spec.sample.schema_handler))
        ds = ds.assemble(partial(LLMSampleAssembler, spec.sample))
        ds = ds.assemble(LLMSampleGuard)
        ds = ds.assemble(partial(spec.packing.assembler_cls or LLMPackingAssembler, spec.packing))
        ds = ds.map(methodcaller("to_model_inputs"))
        ds = ds.assemble(partial(LLMModelInputGuard, ignore_index=spec.sample.tokenization_handler.ignore_index,
                                 verbose=False))
        return ds

    def build_collator(self, spec: LLMDataSpec) -> LLMBatchCollator:
        pad = getattr(spec.sample.tokenization_handler.tokenizer, "pad_token_id", None)
        if pad is None:
            raise ValueError("Tokenizer must expose a pad_token_id to build an LLM collator.")
        return LLMBatchCollator(pad_token_id=int(pad), ignore_index=spec.sample.tokenization_handler.ignore_index)

    def build_dataloader(self, dataset: Dataset, spec: LLMDataSpec, *, device: torch.device | None = None):
        ld = spec.loader
        pin = ld.pin_memory if ld.pin_memory is not None else (device is not None and device.type == "cuda")
        return TorchLoader(dataset, num_workers=ld.num_workers, pin_memory=pin,
                           persistent_workers=ld.persistent_workers,
                           multiprocessing_context=ld.multiprocessing_context).batch(
            batch_size=ld.batch_size, drop_last=ld.drop_last, collate_fn=self.build_collator(spec))

    def to_device(self, batch: ModelInputs, device: torch.device) -> ModelInputs:
        return {k: (v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v) for k, v in batch.items()}


__all__ = ["IGNORE_INDEX", "LLMBatchCollator", "LLMDataKit", "ModelInputs"]
