"""Text samples and fixed-length packs.

Public API of the reference's ``mvp_engine/kit/llm/data/sample.py:20-241``:
``LLMSample`` (a raw row that tokenises on first use and can split into
max-length chunks), ``LLMSampleAssembler`` (row -> chunks) and ``LLMPack`` (one
packed chunk of the token stream).

Here a sample is a raw row plus at most one :class:`TokenChunk`.  A row that
has not been tokenised has no chunk yet; tokenising it computes every chunk
once (schema normalisation, then the tokenisation handler) and keeps the first;
``to_chunks`` turns each chunk into its own sample.  A row that fails to
normalise or tokenise becomes an empty sample, which the guards drop.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from ....data import Assembler, stable_fingerprint
from ....utils.log import simple_info
from .spec import LLMSampleSpec


@dataclass(frozen=True)
class TokenChunk:
    """Aligned token fields of one chunk plus its metadata (schema fields and ``chunk_index``)."""

    input_ids: list[int]
    labels: list[int]
    attention_mask: list[int]
    metadata: dict[str, Any] = field(default_factory=dict)

    def __len__(self) -> int:
        return len(self.input_ids)


_EMPTY = TokenChunk([], [], [])
_OWN_ATTRS = frozenset({"_raw", "schema_handler", "tokenization_handler", "_chunk"})


def _long(values: Sequence[int]) -> torch.Tensor:
    return torch.tensor(list(values), dtype=torch.long)


class LLMSample:
    """A raw row; its token fields are computed on first access.

    Fields of the raw row read and write as attributes (``sample.id``)."""

    def __init__(self, raw: Mapping[str, Any], *, schema_handler, tokenization_handler,
                 metadata: Optional[Mapping[str, Any]] = None, input_ids: Optional[Sequence[int]] = None,
                 labels: Optional[Sequence[int]] = None, attention_mask: Optional[Sequence[int]] = None) -> None:
        chunk = None
        if input_ids is not None:
            chunk = TokenChunk(list(input_ids), list(labels or []), list(attention_mask or []), dict(metadata or {}))
        self.__dict__.update(_raw=dict(raw), schema_handler=schema_handler,
                             tokenization_handler=tokenization_handler, _chunk=chunk)

    # raw-row fields as attributes
    def __getattr__(self, name: str) -> Any:
        raw = self.__dict__.get("_raw", {})
        if name in raw:
            return raw[name]
        raise AttributeError(name)

    def __setattr__(self, name: str, value: Any) -> None:
        if name in _OWN_ATTRS:
            self.__dict__[name] = value
        else:
            self.__dict__["_raw"][name] = value

    @classmethod
    def from_row(cls, row: Mapping[str, Any], *, sample_spec: LLMSampleSpec) -> "LLMSample":
        return cls(row, schema_handler=sample_spec.schema_handler,
                   tokenization_handler=sample_spec.tokenization_handler)

    @classmethod
    def from_tokens(cls, row: Mapping[str, Any], *, sample_spec: LLMSampleSpec, metadata: Mapping[str, Any],
                    input_ids: Sequence[int], labels: Sequence[int],
                    attention_mask: Sequence[int]) -> "LLMSample":
        return cls(row, schema_handler=sample_spec.schema_handler,
                   tokenization_handler=sample_spec.tokenization_handler, metadata=metadata,
                   input_ids=input_ids, labels=labels, attention_mask=attention_mask)

    def _compute_chunks(self) -> list[TokenChunk]:
        try:
            segments, meta = self.schema_handler.normalize(self._raw)
            pieces = self.tokenization_handler.tokenize(segments)
        except Exception as exc:  # noqa: BLE001 - a malformed row becomes an empty sample
            simple_info(str(exc), level="debug")
            return []
        return [TokenChunk(list(ids), list(lab), list(mask), {**meta, "chunk_index": k})
                for k, (ids, lab, mask) in enumerate(pieces)]

    def _tokens(self) -> TokenChunk:
        if self._chunk is None:
            chunks = self._compute_chunks()
            self._chunk = chunks[0] if chunks else _EMPTY
        return self._chunk

    @property
    def _metadata(self) -> dict[str, Any]:
        return self._tokens().metadata

    @property
    def input_ids(self) -> list[int]:
        return self._tokens().input_ids

    @property
    def labels(self) -> list[int]:
        return self._tokens().labels

    @property
    def attention_mask(self) -> list[int]:
        return self._tokens().attention_mask

    @property
    def token_length(self) -> int:
        return len(self._tokens())

    def tokenize(self) -> "LLMSample":
        """Compute the token fields (the row's first chunk) if they are not there yet."""
        self._tokens()
        return self

    def to_chunks(self) -> list["LLMSample"]:
        """One sample per max-length chunk of this row; [] for an empty or malformed row."""
        if self._chunk is not None:
            return [self] if len(self._chunk) else []
        out = []
        for chunk in self._compute_chunks():
            piece = LLMSample(self._raw, schema_handler=self.schema_handler,
                              tokenization_handler=self.tokenization_handler)
            piece._chunk = chunk
            out.append(piece)
        return out

    def to_model_inputs(self) -> dict[str, Any]:
        tok = self._tokens()
        return {"input_ids": _long(tok.input_ids), "attention_mask": _long(tok.attention_mask),
                "labels": _long(tok.labels)}

    def set_empty(self) -> None:
        """Mark the sample empty so the guards drop it."""
        self._chunk = _EMPTY


class LLMSampleAssembler(Assembler):
    """Raw row -> its tokenised chunks (stateless)."""

    def __init__(self, sample_spec: LLMSampleSpec, assemble_context: Any = None) -> None:
        self.sample_spec = sample_spec

    def push(self, row: dict[str, Any]) -> list[LLMSample]:
        return LLMSample.from_row(row, sample_spec=self.sample_spec).to_chunks()

    def fingerprint(self) -> str:
        spec = self.sample_spec
        return stable_fingerprint([type(self).__name__, repr(spec.schema_handler),
                                   repr(spec.tokenization_handler)])


_PACK_TENSORS = ("input_ids", "attention_mask", "labels", "pack_segment_ids")


@dataclass(frozen=True)
class LLMPack:
    """One fixed-length chunk of the packed token stream."""

    input_ids: list[int]
    labels: list[int]
    attention_mask: list[int]
    pack_segment_ids: list[int]
    source_sample_num: int
    position_ids: Optional[list[int]] = None

    def to_model_inputs(self) -> dict[str, Any]:
        out: dict[str, Any] = {name: _long(getattr(self, name)) for name in _PACK_TENSORS}
        out["source_sample_num"] = int(self.source_sample_num)
        if self.position_ids is not None:
            out["position_ids"] = _long(self.position_ids)
        return out
