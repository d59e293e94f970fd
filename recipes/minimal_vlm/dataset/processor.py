"""Processor of the minimal VLM recipe (reference: recipes/minimal_vlm/dataset/processor.py): the HF
processor when it is available locally, else the engine's built-in Qwen-VL processor."""

from __future__ import annotations

from mvp_engine.kit.mllm import MLLMDataKit


def build_qwen3_vl_processor(model_config, synthetic: bool = False):
    name = "synthetic" if synthetic else model_config.pretrained_model_name_or_path
    return MLLMDataKit().build_processor(name, image_max_pixels=model_config.image_max_pixels)
