"""Text-LM data kit: tokenizer, streaming dataset, collator and loader.

Public API of the reference's ``LLMDataKit`` (``mvp_engine/kit/llm/data/data.py:25-140``).  The
order of the pipeline stages is part of that contract (raw-row guard -> tokenised chunks ->
sample guard -> packer -> model inputs -> model-input guard); here the pipeline is a table of
stages folded onto the source, on this repository's streaming runtime (``mvp_engine.data``).
Tokenizers come from Hugging Face files when they are available offline and otherwise from
the synthetic tokenizer, so the kit also runs without any downloaded assets.
"""

from __future__ import annotations

import functools
from functools import partial
from operator import methodcaller
from typing import Any, Callable, Optional

import torch

from ....data import Dataset, RuntimeContext, SyntheticTokenizer, TorchLoader
from .collator import LLMBatchCollator
from .guard import LLMModelInputGuard, LLMRawRowGuard, LLMSampleGuard
from .packing import LLMPackingAssembler
from .sample import LLMSampleAssembler
from .spec import LLMDataSpec, LLMDistributionSpec
from .types import ModelInputs

IGNORE_INDEX = -100


def _hf_tokenizer(name: str, trust_remote_code: bool, **kwargs: Any) -> Any:
    from transformers import AutoTokenizer

    return AutoTokenizer.from_pretrained(name, trust_remote_code=trust_remote_code, **kwargs)


class LLMDataKit:
    def build_distribution_spec(self, *, parallel_mesh) -> LLMDistributionSpec:
        return LLMDistributionSpec(device_mesh=parallel_mesh.device_mesh, dp_dims=parallel_mesh.dp.dim_names or None)

    def build_tokenizer(self, pretrained_model_name_or_path: str, *, trust_remote_code: bool = True,
                        padding_side: str = "right", pad_token_fallback_to_eos: bool = True, **kwargs: Any) -> Any:
        """The Hugging Face tokenizer when its files can be loaded, else :class:`SyntheticTokenizer`."""
        name = pretrained_model_name_or_path
        tok = None
        if not name.startswith("synthetic"):
            try:
                tok = _hf_tokenizer(name, trust_remote_code, **kwargs)
            except Exception:  # noqa: BLE001 - no files offline: fall back to the synthetic vocabulary
                tok = None
        if tok is None:
            return SyntheticTokenizer()
        tok.padding_side = padding_side
        if pad_token_fallback_to_eos and tok.pad_token_id is None and tok.eos_token is not None:
            tok.pad_token = tok.eos_token
        return tok

    @staticmethod
    def _context(spec: LLMDataSpec) -> RuntimeContext:
        seed = spec.source.seed
        d = spec.distribution
        if d is not None and d.device_mesh is not None and d.dp_dims is not None:
            return RuntimeContext.from_runtime(seed=seed, device_mesh=d.device_mesh, dp_dims=d.dp_dims)
        return RuntimeContext.from_runtime(seed=seed)

    @staticmethod
    def _stages(spec: LLMDataSpec) -> list[tuple[str, Callable]]:
        ignore = spec.sample.tokenization_handler.ignore_index
        packer = spec.packing.assembler_cls or LLMPackingAssembler
        return [
            ("assemble", partial(LLMRawRowGuard, schema_handler=spec.sample.schema_handler)),
            ("assemble", partial(LLMSampleAssembler, spec.sample)),
            ("assemble", LLMSampleGuard),
            ("assemble", partial(packer, spec.packing)),
            ("map", methodcaller("to_model_inputs")),
            ("assemble", partial(LLMModelInputGuard, ignore_index=ignore, verbose=False)),
        ]

    def build_dataset(self, spec: LLMDataSpec) -> Dataset:
        src = spec.source
        source = Dataset.from_source(src.dataset_source, src.dataset_path, context=self._context(spec),
                                     resample=src.resample, shuffle_mode=src.shuffle_mode)
        return functools.reduce(lambda ds, stage: getattr(ds, stage[0])(stage[1]), self._stages(spec), source)

    def build_collator(self, spec: LLMDataSpec) -> LLMBatchCollator:
        handler = spec.sample.tokenization_handler
        pad = getattr(handler.tokenizer, "pad_token_id", None)
        if pad is None:
            raise ValueError("Tokenizer must expose a pad_token_id to build an LLM collator.")
        return LLMBatchCollator(pad_token_id=int(pad), ignore_index=handler.ignore_index)

    def build_dataloader(self, dataset: Dataset, spec: LLMDataSpec, *, device: Optional[torch.device] = None):
        opts = spec.loader
        pin = opts.pin_memory
        if pin is None:  # default: pin host batches when they feed a GPU
            pin = device is not None and device.type == "cuda"
        loader = TorchLoader(dataset, num_workers=opts.num_workers, pin_memory=pin,
                             persistent_workers=opts.persistent_workers,
                             multiprocessing_context=opts.multiprocessing_context)
        return loader.batch(batch_size=opts.batch_size, drop_last=opts.drop_last, collate_fn=self.build_collator(spec))

    def to_device(self, batch: ModelInputs, device: torch.device) -> ModelInputs:
        return {k: v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v for k, v in batch.items()}


__all__ = ["IGNORE_INDEX", "LLMBatchCollator", "LLMDataKit", "ModelInputs"]
