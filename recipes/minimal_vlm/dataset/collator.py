"""Padding collator of the minimal VLM recipe (reference: recipes/minimal_vlm/dataset/collator.py:11-62)."""

from __future__ import annotations

import torch
from torch.nn.utils.rnn import pad_sequence

from .types import ModelInputs


class MinimalVLMCollator:
    def __init__(self, pad_token_id: int, *, ignore_index: int = -100) -> None:
        self.pad_token_id = int(pad_token_id)
        self.ignore_index = int(ignore_index)

    def __call__(self, batch: list[dict]) -> ModelInputs:
        out: ModelInputs = {
            "input_ids": pad_sequence([s["input_ids"] for s in batch], batch_first=True,
                                      padding_value=self.pad_token_id),
            "attention_mask": pad_sequence([s["attention_mask"] for s in batch], batch_first=True, padding_value=0),
            "labels": pad_sequence([s["labels"] for s in batch], batch_first=True, padding_value=self.ignore_index),
        }
        px = [s["pixel_values"] for s in batch if s.get("pixel_values") is not None]
        if px:
            out["pixel_values"] = torch.cat(px, dim=0)
            out["image_grid_thw"] = torch.cat([s["image_grid_thw"] for s in batch
                                               if s.get("image_grid_thw") is not None], dim=0)
        return out
