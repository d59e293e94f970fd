"""Qwen3-VL model patches (reference: recipes/qwen3_vl/model/qwen3_vl.py:11-175).

* ``patch_qwen3vl_conv3d``: the reference swaps the vision patch-embed Conv3d
  for an fp32 ``F.linear`` over flattened patches.  The engine's
  ``Qwen3VLVisionPatchEmbed`` already is a linear over flattened patches with
  fp32-accurate products (three bf16 tensor-core GEMMs over hi/lo splits), so
  the patch only marks the model.
* ``patch_qwen3vl_model_flops``: binds ``calculate_model_flops`` (LM + ViT +
  mergers, frozen parts forward-only) as the model's FLOPs method.
"""

from __future__ import annotations

from types import MethodType
from typing import Any, Optional

import torch

from mvp_engine.models.qwen3_vl import Qwen3VLForConditionalGeneration


def calculate_model_flops(self, *, batch_size: int, seq_len: int, attention_mask: Optional[torch.Tensor] = None,
                          attention_token_pairs: Optional[int] = None, image_grid_thw: Optional[torch.Tensor] = None,
                          is_training: bool = True, freeze_vit: bool = False, freeze_projector: bool = False,
                          freeze_llm: bool = False, **unused: Any) -> float:
    if attention_token_pairs is None and attention_mask is not None:
        pairs = 0
        for row in attention_mask.detach().to("cpu"):
            r = row[row > 0].long()
            if r.numel():
                pairs += int(torch.bincount(r).pow(2).sum())
        attention_token_pairs = pairs
    return Qwen3VLForConditionalGeneration.calculate_model_flops(
        self, batch_size=batch_size, seq_len=seq_len, attention_token_pairs=attention_token_pairs,
        image_grid_thw=image_grid_thw, is_training=is_training, freeze_llm=freeze_llm, freeze_vit=freeze_vit,
        freeze_projector=freeze_projector)


def patch_qwen3vl_conv3d(model):
    embed = model.model.visual.patch_embed
    if not isinstance(getattr(embed, "proj", None), (torch.nn.Conv3d, torch.nn.Linear)):
        raise TypeError("Qwen3-VL patch embed is expected to hold a Conv3d / Linear projection")
    model._mvp_patch_embed_fp32_linear = True
    return model


def patch_qwen3vl_model_flops(model):
    model.calculate_model_flops = MethodType(calculate_model_flops, model)
    return model
