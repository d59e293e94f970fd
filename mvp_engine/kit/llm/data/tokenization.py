"""Segment tokenisation with per-segment loss flags (reference: mvp_engine/kit/llm/data/tokenization.py:14-55)."""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

from .types import LLMSegment

TokenizedFields = tuple[list[int], list[int], list[int]]


@dataclass(slots=True)
class LLMTokenizationHandler:
    """Tokenise segments, label supervised ones, append EOS, split into ``max_seq_len`` chunks."""

    tokenizer: Any
    max_seq_len: int
    ignore_index: int = -100
    add_eos: bool = True

    def __post_init__(self) -> None:
        if self.max_seq_len <= 0:
            raise ValueError("LLMTokenizationHandler.max_seq_len must be positive.")

    def segment_ids(self, seg: LLMSegment) -> list[int]:
        if seg.type == "tokens":
            return [int(t) for t in seg.value]
        if seg.type != "text":
            raise ValueError(f"Unsupported LLM segment type: {seg.type!r}.")
        if not isinstance(seg.value, str):
            raise TypeError("LLM text segment value must be a string.")
        return list(self.tokenizer(seg.value, add_special_tokens=False)["input_ids"])

    def tokenize(self, segments: Sequence[LLMSegment]) -> list[TokenizedFields]:
        ids: list[int] = []
        labels: list[int] = []
        for seg in segments:
            part = self.segment_ids(seg)
            ids.extend(part)
            labels.extend(part if seg.loss else [self.ignore_index] * len(part))
        if self.add_eos and ids:
            eos = getattr(self.tokenizer, "eos_token_id", None)
            if eos is None:
                raise ValueError("Tokenizer has no eos_token_id; required when add_eos=True.")
            ids.append(int(eos))
            labels.append(int(eos) if (segments[-1].loss if segments else True) else self.ignore_index)
        out: list[TokenizedFields] = []
        for s in range(0, len(ids), self.max_seq_len):
            chunk = ids[s:s + self.max_seq_len]
            if chunk:
                out.append((chunk, labels[s:s + self.max_seq_len], [1] * len(chunk)))
        return out


@dataclass(slots=True)
class LLMPretrainTextTokenizationHandler(LLMTokenizationHandler):
    """Full-token-loss pretraining tokenisation."""
