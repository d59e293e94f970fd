"""OpenBee engine (reference: recipes/openbee/engine/openbee_engine.py): the Qwen3-VL engine whose
training loader additionally maps ``MLLMTextOnlyBatchGuard`` over the batches, so a text-only batch
still carries one (dummy, unsupervised) image and every rank runs the vision tower each step —
required when ViT / projector parameters are sharded or all-reduced across ranks."""

from __future__ import annotations

from mvp_engine.engine import ENGINE_REGISTRY
from mvp_engine.kit.mllm import MLLMTextOnlyBatchGuard, QwenImageHandler
from recipes.qwen3_vl.engine.qwen3_vl_engine import Qwen3VLEngine

from ..configs.schema import OpenBeeConfig


@ENGINE_REGISTRY.register()
class OpenBeeEngine(Qwen3VLEngine):
    ConfigClass = OpenBeeConfig
    config: OpenBeeConfig

    def prepare_dataloader(self, workflow: str = "train"):
        loader = super().prepare_dataloader(workflow)
        if loader is None:
            return None
        handler = QwenImageHandler()
        tok = self.processor.tokenizer
        return loader.map(MLLMTextOnlyBatchGuard(dummy_inputs=handler.build_dummy_inputs(self.processor),
                                                 media_keys=handler.OUTPUT_TENSOR_KEYS,
                                                 pad_token_id=int(tok.pad_token_id), ignore_index=-100))
