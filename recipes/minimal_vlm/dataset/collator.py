"""Padding collator of the minimal VLM recipe.

Behaviour of the reference's ``recipes/minimal_vlm/dataset/collator.py:11-62``: right-pad
``input_ids`` with the pad id, ``attention_mask`` with 0 and ``labels`` with the ignore index to
the longest sample of the batch; concatenate the samples' ``pixel_values`` and
``image_grid_thw`` along the image axis.  The padded batch is built by filling one
preallocated tensor per field.
"""

from __future__ import annotations

from typing import Sequence

import torch

from .types import ModelInputs


def _right_padded(rows: Sequence[torch.Tensor], fill: int) -> torch.Tensor:
    width = max(r.numel() for r in rows)
    out = torch.full((len(rows), width), fill, dtype=rows[0].dtype)
    for i, r in enumerate(rows):
        out[i, : r.numel()] = r
    return out


class MinimalVLMCollator:
    def __init__(self, pad_token_id: int, *, ignore_index: int = -100) -> None:
        self.pad_token_id = int(pad_token_id)
        self.ignore_index = int(ignore_index)

    def __call__(self, batch: list[dict]) -> ModelInputs:
        fills = {"input_ids": self.pad_token_id, "attention_mask": 0, "labels": self.ignore_index}
        out: ModelInputs = {key: _right_padded([s[key] for s in batch], fill) for key, fill in fills.items()}
        for key in ("pixel_values", "image_grid_thw"):
            parts = [s[key] for s in batch if s.get(key) is not None]
            if parts:
                out[key] = torch.cat(parts, dim=0)
        return out
