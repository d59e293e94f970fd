"""Tokenised samples and fixed-length packs (reference: mvp_engine/kit/llm/data/sample.py:20-241)."""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from typing import Any, Optional

import torch

from ....data import Assembler, stable_fingerprint
from ....utils.log import simple_info
from .spec import LLMSampleSpec


class LLMSample:
    """One row (or one max-length chunk of it) with lazily materialised token fields.

    Raw-row fields read and write as attributes (``sample.id``).
    """

    __slots__ = ("_raw", "schema_handler", "tokenization_handler", "_metadata", "_input_ids", "_labels",
                 "_attention_mask")

    def __init__(self, raw: Mapping[str, Any], *, schema_handler, tokenization_handler,
                 metadata: Optional[Mapping[str, Any]] = None, input_ids: Optional[Sequence[int]] = None,
                 labels: Optional[Sequence[int]] = None, attention_mask: Optional[Sequence[int]] = None) -> None:
        object.__setattr__(self, "_raw", dict(raw))
        object.__setattr__(self, "schema_handler", schema_handler)
        object.__setattr__(self, "tokenization_handler", tokenization_handler)
        object.__setattr__(self, "_metadata", dict(metadata or {}))
        object.__setattr__(self, "_input_ids", list(input_ids) if input_ids is not None else None)
        object.__setattr__(self, "_labels", list(labels) if labels is not None else None)
        object.__setattr__(self, "_attention_mask", list(attention_mask) if attention_mask is not None else None)

    def __getattr__(self, name: str) -> Any:
        raw = object.__getattribute__(self, "_raw")
        if name in raw:
            return raw[name]
        raise AttributeError(name)

    def __setattr__(self, name: str, value: Any) -> None:
        if name in LLMSample.__slots__:
            object.__setattr__(self, name, value)
        else:
            self._raw[name] = value

    @classmethod
    def from_row(cls, row: Mapping[str, Any], *, sample_spec: LLMSampleSpec) -> "LLMSample":
        return cls(row, schema_handler=sample_spec.schema_handler,
                   tokenization_handler=sample_spec.tokenization_handler)

    @classmethod
    def from_tokens(cls, row, *, sample_spec: LLMSampleSpec, metadata, input_ids, labels, attention_mask):
        return cls(row, schema_handler=sample_spec.schema_handler,
                   tokenization_handler=sample_spec.tokenization_handler, metadata=metadata, input_ids=input_ids,
                   labels=labels, attention_mask=attention_mask)

    @property
    def input_ids(self) -> list[int]:
        self.tokenize()
        return self._input_ids or []

    @property
    def labels(self) -> list[int]:
        self.tokenize()
        return self._labels or []

    @property
    def attention_mask(self) -> list[int]:
        self.tokenize()
        return self._attention_mask or []

    @property
    def token_length(self) -> int:
        return len(self.input_ids)

    def tokenize(self) -> "LLMSample":
        if self._input_ids is not None:
            return self
        chunks = self.to_chunks()
        if not chunks:
            self.set_empty()
            return self
        first = chunks[0]
        self._metadata = dict(first._metadata)
        self._input_ids, self._labels, self._attention_mask = first._input_ids, first._labels, first._attention_mask
        return self

    def to_chunks(self) -> list["LLMSample"]:
        if self._input_ids is not None:
            return [self] if self._input_ids else []
        try:
            segments, meta = self.schema_handler.normalize(self._raw)
            pieces = self.tokenization_handler.tokenize(segments)
        except Exception as exc:  # malformed rows become empty samples; guards drop them
            simple_info(str(exc), level="debug")
            return []
        return [LLMSample(self._raw, schema_handler=self.schema_handler,
                          tokenization_handler=self.tokenization_handler, metadata={**meta, "chunk_index": i},
                          input_ids=a, labels=b, attention_mask=c) for i, (a, b, c) in enumerate(pieces)]

    def to_model_inputs(self) -> dict[str, Any]:
        return {"input_ids": torch.tensor(self.input_ids, dtype=torch.long),
                "attention_mask": torch.tensor(self.attention_mask, dtype=torch.long),
                "labels": torch.tensor(self.labels, dtype=torch.long)}

    def set_empty(self) -> None:
        self._input_ids, self._labels, self._attention_mask = [], [], []


class LLMSampleAssembler(Assembler):
    """Raw row -> one or more tokenised chunks."""

    def __init__(self, sample_spec: LLMSampleSpec, assemble_context: Any = None) -> None:
        self.sample_spec = sample_spec

    def push(self, row: dict[str, Any]) -> list[LLMSample]:
        return LLMSample.from_row(row, sample_spec=self.sample_spec).to_chunks()

    def fingerprint(self) -> str:
        return stable_fingerprint({"kind": type(self).__name__, "schema": repr(self.sample_spec.schema_handler),
                                   "tok": type(self.sample_spec.tokenization_handler).__name__})


@dataclass(frozen=True, slots=True)
class LLMPack:
    """One fixed-length chunk of the packed token stream."""

    input_ids: list[int]
    labels: list[int]
    attention_mask: list[int]
    pack_segment_ids: list[int]
    source_sample_num: int
    position_ids: Optional[list[int]] = None

    def to_model_inputs(self) -> dict[str, Any]:
        out: dict[str, Any] = {
            "input_ids": torch.tensor(self.input_ids, dtype=torch.long),
            "attention_mask": torch.tensor(self.attention_mask, dtype=torch.long),
            "labels": torch.tensor(self.labels, dtype=torch.long),
            "pack_segment_ids": torch.tensor(self.pack_segment_ids, dtype=torch.long),
            "source_sample_num": int(self.source_sample_num),
        }
        if self.position_ids is not None:
            out["position_ids"] = torch.tensor(self.position_ids, dtype=torch.long)
        return out
