"""Multimodal samples and packs (reference: mvp_engine/kit/mllm/data/sample.py:20-306)."""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from typing import Any, Optional

import torch

from ....utils.log import simple_info
from .media import is_empty_model_sample
from .spec import MLLMSampleSpec


class MLLMSample:
    """One row: lazily normalised -> rendered -> tokenised; media loaded on demand."""

    __slots__ = ("_raw", "schema_handler", "media_handler", "tokenization_handler", "segments", "media_slots",
                 "metadata", "_input_ids", "_labels", "_attention_mask", "media")

    def __init__(self, raw: Mapping[str, Any], spec: Optional[MLLMSampleSpec] = None, *, schema_handler: Any = None,
                 media_handler: Any = None, tokenization_handler: Any = None) -> None:
        """The three handlers, given directly (the reference's form) or through an ``MLLMSampleSpec``."""
        if spec is not None:
            schema_handler = schema_handler or spec.schema_handler
            media_handler = media_handler or spec.media_handler
            tokenization_handler = tokenization_handler or spec.tokenization_handler
        if schema_handler is None or media_handler is None or tokenization_handler is None:
            raise ValueError("MLLMSample needs schema_handler, media_handler and tokenization_handler")
        object.__setattr__(self, "_raw", dict(raw))
        object.__setattr__(self, "schema_handler", schema_handler)
        object.__setattr__(self, "media_handler", media_handler)
        object.__setattr__(self, "tokenization_handler", tokenization_handler)
        for k in ("segments", "media_slots", "_input_ids", "_labels", "_attention_mask", "media"):
            object.__setattr__(self, k, None)
        object.__setattr__(self, "metadata", {})

    def __getattr__(self, name: str) -> Any:
        raw = object.__getattribute__(self, "_raw")
        if name in raw:
            return raw[name]
        raise AttributeError(name)

    def __setattr__(self, name: str, value: Any) -> None:
        if name in MLLMSample.__slots__:
            object.__setattr__(self, name, value)
        else:
            self._raw[name] = value

    @classmethod
    def from_row(cls, row: Mapping[str, Any], *, sample_spec: MLLMSampleSpec) -> "MLLMSample":
        return cls(row, sample_spec)

    def tokenize(self) -> "MLLMSample":
        if self._input_ids is not None:
            return self
        try:
            segs, slots, meta = self.schema_handler.normalize(self._raw)
            ids, labels, am = self.tokenization_handler.tokenize(self.media_handler.render(segs, slots))
            self.segments, self.media_slots, self.metadata = segs, slots, meta
            self._input_ids, self._labels, self._attention_mask = ids, labels, am
        except Exception as exc:
            simple_info(str(exc), level="debug")
            self.set_empty()
        return self

    @property
    def input_ids(self) -> list[int]:
        return self.tokenize()._input_ids or []

    @property
    def labels(self) -> list[int]:
        return self.tokenize()._labels or []

    @property
    def attention_mask(self) -> list[int]:
        return self.tokenize()._attention_mask or []

    @property
    def token_length(self) -> int:
        return len(self.input_ids)

    def load_media(self) -> "MLLMSample":
        if self.media is None:
            self.tokenize()
            self.media = self.media_handler.load(self, self.media_slots or []) if self.media_slots else {}
        return self

    def to_model_inputs(self) -> dict[str, Any]:
        self.load_media()
        if is_empty_model_sample(self.media or {}):
            return {"__empty__": True}
        out = {"input_ids": torch.tensor(self.input_ids, dtype=torch.long),
               "attention_mask": torch.tensor(self.attention_mask, dtype=torch.long),
               "labels": torch.tensor(self.labels, dtype=torch.long)}
        out.update(self.media or {})
        return out

    def set_empty(self) -> None:
        self._input_ids, self._labels, self._attention_mask = [], [], []
        self.segments, self.media_slots = [], []


class MLLMPack(list):
    """Samples packed into one sequence (documents keep their own segment id)."""

    def __init__(self, samples: Sequence[MLLMSample]) -> None:
        super().__init__(samples)

    @property
    def source_sample_num(self) -> int:
        return len(self)

    @property
    def token_length(self) -> int:
        return sum(s.token_length for s in self)

    def to_model_inputs(self, *, load_media: bool = True) -> dict[str, Any]:
        parts = [s.to_model_inputs() for s in self]
        if any(p.get("__empty__") for p in parts):
            return {"__empty__": True}
        ids = torch.cat([p["input_ids"] for p in parts])
        seg = torch.cat([torch.full_like(p["input_ids"], i + 1) for i, p in enumerate(parts)])
        out = {"input_ids": ids, "attention_mask": torch.cat([p["attention_mask"] for p in parts]),
               "labels": torch.cat([p["labels"] for p in parts]), "pack_segment_ids": seg,
               "source_sample_num": len(parts)}
        if load_media and self:
            out.update(self[0].media_handler.merge_pack(parts))
        return out
