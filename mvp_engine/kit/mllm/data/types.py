"""Multimodal data types (reference: mvp_engine/kit/mllm/data/types.py:1-71)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, NotRequired, TypedDict

import torch


@dataclass(frozen=True, slots=True)
class MLLMMediaSlot:
    """A media reference of one sample: ``field[index]`` of the raw row holds the media."""

    media_id: str
    media_type: str
    field: str
    index: int | None = None
    metadata: dict[str, Any] = field(default_factory=dict)


@dataclass(frozen=True, slots=True)
class MLLMSegment:
    """Ordered text (``type="text"``) or media (``type`` = media type, ``value`` = media id) segment."""

    type: str
    loss: bool
    value: Any


class ModelInputs(TypedDict):
    input_ids: torch.Tensor
    attention_mask: torch.Tensor | None
    labels: torch.Tensor
    pack_segment_ids: torch.Tensor
    source_sample_num: torch.Tensor
    num_input_tokens: torch.Tensor
    num_loss_tokens: torch.Tensor
    num_source_samples: torch.Tensor
    pixel_values: NotRequired[torch.Tensor]
    pixel_values_videos: NotRequired[torch.Tensor]
    image_grid_thw: NotRequired[torch.Tensor]
    video_grid_thw: NotRequired[torch.Tensor]
    position_ids: NotRequired[torch.Tensor]
    cu_seq_lens_q: NotRequired[torch.Tensor]
    cu_seq_lens_k: NotRequired[torch.Tensor]
    max_length_q: NotRequired[int]
    max_length_k: NotRequired[int]
    total_tokens: NotRequired[int]
    effective_tokens: NotRequired[int]
