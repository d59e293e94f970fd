"""Segment tokenisation for text samples.

Public API of the reference's ``mvp_engine/kit/llm/data/tokenization.py:14-55``:
``tokenize(segments)`` returns ``(input_ids, labels, attention_mask)`` chunks of
at most ``max_seq_len`` tokens.  Behaviour kept: segments are tokenised without
special tokens; a segment with ``loss=False`` gets ``ignore_index`` labels; one
EOS token closes a non-empty sample and is supervised when the last segment is.
Added: ``"tokens"`` segments carry ids already (synthetic and pre-tokenised data).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

from .types import LLMSegment

TokenizedFields = tuple[list[int], list[int], list[int]]


def _windows(n: int, size: int) -> range:
    return range(0, n, size)


@dataclass
class LLMTokenizationHandler:
    """Tokenise segments, mask unsupervised ones, close with EOS, cut into ``max_seq_len`` chunks."""

    tokenizer: Any
    max_seq_len: int
    ignore_index: int = -100
    add_eos: bool = True

    def __post_init__(self) -> None:
        if self.max_seq_len <= 0:
            raise ValueError("LLMTokenizationHandler.max_seq_len must be positive.")

    def segment_ids(self, seg: LLMSegment) -> list[int]:
        kind = seg.type
        if kind == "tokens":
            return list(map(int, seg.value))
        if kind != "text":
            raise ValueError(f"Unsupported LLM segment type: {kind!r}.")
        if not isinstance(seg.value, str):
            raise TypeError("LLM text segment value must be a string.")
        return list(self.tokenizer(seg.value, add_special_tokens=False)["input_ids"])

    def _eos(self) -> int:
        eos = getattr(self.tokenizer, "eos_token_id", None)
        if eos is None:
            raise ValueError("Tokenizer has no eos_token_id; required when add_eos=True.")
        return int(eos)

    def tokenize(self, segments: Sequence[LLMSegment]) -> list[TokenizedFields]:
        parts = [(self.segment_ids(seg), bool(seg.loss)) for seg in segments]
        ids = [t for toks, _ in parts for t in toks]
        labels = [t if supervised else self.ignore_index for toks, supervised in parts for t in toks]
        if ids and self.add_eos:
            eos = self._eos()
            last_supervised = parts[-1][1] if parts else True
            ids.append(eos)
            labels.append(eos if last_supervised else self.ignore_index)
        n = self.max_seq_len
        return [(ids[s:s + n], labels[s:s + n], [1] * len(ids[s:s + n])) for s in _windows(len(ids), n)]


@dataclass
class LLMPretrainTextTokenizationHandler(LLMTokenizationHandler):
    """Pretraining: every token supervised (segments come with ``loss=True``)."""
