"""Row -> training sample for the minimal VLM recipe (reference: recipes/minimal_vlm/dataset/preprocess.py:30-534).

Same behaviour as the reference's hand-rolled preprocessing, expressed with the multimodal kit's
handlers: the chat (or synthetic token) schema gives text segments and image slots; images are
smart-resized to multiples of 32 px within the processor's pixel bounds and patchified; every
image placeholder expands to ``t*h*w/4`` image tokens; only assistant text is supervised (prompt,
template and image tokens get label -100); a sample whose truncation to ``max_length`` would cut
image tokens is dropped instead of corrupting the image/text alignment.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from mvp_engine.kit.mllm import MLLMSample, MLLMSampleSpec, QwenVLChatSchemaHandler, QwenVLMediaHandler
from mvp_engine.kit.mllm import QwenVLTokenizationHandler
from mvp_engine.kit.mllm.data import SyntheticVLSchemaHandler


def build_sample_spec(processor: Any, max_length: int, synthetic: bool) -> MLLMSampleSpec:
    schema = SyntheticVLSchemaHandler() if synthetic else QwenVLChatSchemaHandler(processor=processor)
    return MLLMSampleSpec(schema_handler=schema, media_handler=QwenVLMediaHandler(processor=processor),
                          tokenization_handler=QwenVLTokenizationHandler(tokenizer=processor.tokenizer,
                                                                         max_seq_len=int(max_length)))


def process_sample(row: dict[str, Any], *, spec: MLLMSampleSpec) -> Optional[dict[str, Any]]:
    """One row -> {input_ids, attention_mask, labels[, pixel_values, image_grid_thw]} or None (dropped)."""
    sample = MLLMSample.from_row(row, sample_spec=spec).load_media()
    if not sample.input_ids:
        return None
    out = {"input_ids": torch.tensor(sample.input_ids, dtype=torch.long),
           "attention_mask": torch.tensor(sample.attention_mask, dtype=torch.long),
           "labels": torch.tensor(sample.labels, dtype=torch.long)}
    media = sample.media or {}
    for key in ("pixel_values", "image_grid_thw"):
        if media.get(key) is not None:
            out[key] = media[key]
    return out
