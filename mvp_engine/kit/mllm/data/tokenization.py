"""Segment tokenisation for multimodal samples (reference: mvp_engine/kit/mllm/data/tokenization.py:12-78).

Text segments are tokenised with their loss flag, media segments become the
handler-rendered placeholder text (never supervised).  A sample longer than
``max_seq_len`` is truncated only inside trailing text: a cut through a media
placeholder drops the sample instead (it would desynchronise image tokens and
image features).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Sequence

from .types import MLLMSegment


@dataclass(slots=True)
class MLLMTokenizationHandler:
    tokenizer: Any
    max_seq_len: int
    ignore_index: int = -100
    add_eos: bool = False

    def __post_init__(self) -> None:
        if self.max_seq_len <= 0:
            raise ValueError("MLLMTokenizationHandler.max_seq_len must be positive.")

    def _encode(self, text: str) -> list[int]:
        enc = self.tokenizer(text, add_special_tokens=False)
        return list(enc["input_ids"])

    def tokenize(self, rendered_segments: Sequence[MLLMSegment]) -> tuple[list[int], list[int], list[int]]:
        """``(input_ids, labels, attention_mask)`` of segments whose media values are already rendered to
        placeholder text (``MLLMMediaHandler.render``)."""
        ids: list[int] = []
        labels: list[int] = []
        media_end = 0
        for seg in rendered_segments:
            if seg.type == "tokens":
                part = [int(t) for t in seg.value]
                sup = seg.loss
            else:  # text, or a media segment's placeholder text (never supervised)
                part = self._encode(seg.value)
                sup = seg.loss and seg.type == "text"
            ids += part
            labels += part if sup else [self.ignore_index] * len(part)
            if seg.type not in ("text", "tokens"):
                media_end = len(ids)
        if self.add_eos and ids:
            eos = getattr(self.tokenizer, "eos_token_id", None)
            if eos is not None:
                ids.append(int(eos))
                labels.append(int(eos))
        if len(ids) > self.max_seq_len:
            if media_end > self.max_seq_len:
                raise ValueError("sample.media_truncated")
            ids, labels = ids[: self.max_seq_len], labels[: self.max_seq_len]
        return ids, labels, [1] * len(ids)


@dataclass(slots=True)
class QwenVLTokenizationHandler(MLLMTokenizationHandler):
    """Qwen-VL chat tokenisation (the chat template closes turns; no extra EOS)."""
