"""Media handling contract (reference: mvp_engine/kit/mllm/data/media.py:14-280).

A ``MLLMMediaTypeHandler`` renders a media slot into placeholder text, loads
the media into model tensors, merges them across the samples of a pack and
collates them across a batch.  ``MLLMMediaHandler`` dispatches by media type.
An empty dict with ``__empty__`` marks a sample whose media could not be read;
guards drop it.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Mapping, Sequence

import torch

from .types import MLLMMediaSlot, MLLMSegment


def empty_model_sample() -> dict[str, Any]:
    return {"__empty__": True}


def is_empty_model_sample(sample: dict[str, Any]) -> bool:
    return bool(sample.get("__empty__", False))


@dataclass(frozen=True, slots=True)
class RenderedMedia:
    media_id: str
    media_type: str
    text: str


class MLLMMediaTypeHandler:
    media_type: str = ""
    OUTPUT_TENSOR_KEYS: tuple[str, ...] = ()

    def render(self, slot: MLLMMediaSlot, *, processor: Any, tokenizer: Any) -> RenderedMedia:
        raise NotImplementedError

    def default_token(self, processor: Any) -> str:
        raise NotImplementedError

    def placeholder_aliases(self, processor: Any) -> tuple[str, ...]:
        return (self.default_token(processor),)

    def load(self, slots: list[MLLMMediaSlot], values: list[Any], *, processor: Any) -> dict[str, Any]:
        raise NotImplementedError

    def merge_pack(self, samples: Sequence[dict[str, Any]]) -> dict[str, Any]:
        return self._cat(samples)

    def collate(self, batch: Sequence[dict[str, Any]]) -> dict[str, Any]:
        return self._cat(batch)

    def _cat(self, items: Sequence[dict[str, Any]]) -> dict[str, Any]:
        out = {}
        for key in self.OUTPUT_TENSOR_KEYS:
            ts = [it[key] for it in items if it.get(key) is not None]
            if ts:
                out[key] = torch.cat(ts, dim=0)
        return out


@dataclass
class MLLMMediaHandler:
    processor: Any
    handlers: dict[str, MLLMMediaTypeHandler] = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.handlers = dict(self.handlers)

    @property
    def tokenizer(self) -> Any:
        return getattr(self.processor, "tokenizer", self.processor)

    def render_slots(self, slots: Sequence[MLLMMediaSlot]) -> dict[str, RenderedMedia]:
        """Placeholder text of every media slot, by media id."""
        out = {}
        for s in slots:
            h = self.handlers.get(s.media_type)
            if h is None:
                raise ValueError(f"No media handler for type {s.media_type!r}")
            out[s.media_id] = h.render(s, processor=self.processor, tokenizer=self.tokenizer)
        return out

    def render(self, segments: Sequence[MLLMSegment], media_slots: Sequence[MLLMMediaSlot]) -> list[MLLMSegment]:
        """The segments with every media segment's value (a media id) replaced by its placeholder text;
        media segments keep their media type (the tokenizer never supervises them)."""
        text = self.render_slots(media_slots)
        out = []
        for seg in segments:
            if seg.type in ("text", "tokens"):
                out.append(seg)
            elif seg.value in text:
                out.append(MLLMSegment(seg.type, False, text[seg.value].text))
            else:
                raise ValueError(f"media segment {seg.value!r} has no slot")
        return out

    def load(self, sample: Any, media_slots: Sequence[MLLMMediaSlot]) -> dict[str, Any]:
        out: dict[str, Any] = {}
        by_type: dict[str, list[MLLMMediaSlot]] = {}
        for s in media_slots:
            by_type.setdefault(s.media_type, []).append(s)
        for mtype, slots in by_type.items():
            values = [self._slot_value(sample, s) for s in slots]
            loaded = self.handlers[mtype].load(slots, values, processor=self.processor)
            if is_empty_model_sample(loaded):
                return empty_model_sample()
            out.update(loaded)
        return out

    def merge_pack(self, samples: Sequence[dict[str, Any]]) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for h in self.handlers.values():
            out.update(h.merge_pack(samples))
        return out

    def collate(self, batch: Sequence[dict[str, Any]]) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for h in self.handlers.values():
            out.update(h.collate(batch))
        return out

    @staticmethod
    def _slot_value(sample: Any, slot: MLLMMediaSlot) -> Any:
        raw = sample._raw if hasattr(sample, "_raw") else sample
        v = raw[slot.field]
        v = v[slot.index] if slot.index is not None else v
        if isinstance(v, Mapping) and ("value" in v or slot.media_type in v):  # a `media` column entry
            return v.get("value", v.get(slot.media_type))
        return v
