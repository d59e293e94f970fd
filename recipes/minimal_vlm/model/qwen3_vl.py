"""Model of the minimal VLM recipe (reference: recipes/minimal_vlm/model/qwen3_vl.py:15-48): the
engine's Qwen3-VL (HF names) with the vision tower and its mergers frozen."""

from __future__ import annotations

from typing import Any

from mvp_engine.kit.mllm import MLLMModelKit

MERGER_PREFIXES = ("model.visual.merger.", "model.visual.deepstack_merger_list.")


def apply_freeze_policy(model) -> int:
    """Freeze ``model.visual.*`` (encoder and mergers); returns the number of frozen elements."""
    frozen = 0
    for name, p in model.named_parameters():
        if name.startswith("model.visual.") or name.startswith(MERGER_PREFIXES):
            p.requires_grad = False
            frozen += p.numel()
    return frozen


def build_qwen3_vl_model(model_config: Any, *, seed: int = 42, device=None):
    model = MLLMModelKit().build_model(model_config.pretrained_model_name_or_path,
                                       load_pretrained_model=model_config.load_pretrained_model,
                                       random_init_seed=seed, device=device, **model_config.config_overrides)
    apply_freeze_policy(model)
    return model
