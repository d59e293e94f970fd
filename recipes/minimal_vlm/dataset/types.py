"""Batch type of the minimal VLM recipe (reference: recipes/minimal_vlm/dataset/types.py)."""

from __future__ import annotations

from typing import TypedDict

import torch


class ModelInputs(TypedDict, total=False):
    input_ids: torch.Tensor
    attention_mask: torch.Tensor
    labels: torch.Tensor
    pixel_values: torch.Tensor
    image_grid_thw: torch.Tensor
