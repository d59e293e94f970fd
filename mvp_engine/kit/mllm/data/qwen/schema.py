"""Qwen-VL chat rows -> segments + image slots (reference: mvp_engine/kit/mllm/data/qwen/schema.py:22-332).

Messages may carry content lists with ``{"type": "image", ...}`` items or
``<image>`` placeholders in text; every image becomes an ``MLLMMediaSlot``
(size from ``image_sizes`` / the item's ``height``/``width``) and an image
segment at its position.  User/assistant pairs split into unsupervised prompt
text and supervised response text through the chat template (ChatML when the
tokenizer has none), with the same ``thinking_mode`` rules as the text kit.
"""

from __future__ import annotations

import re
from collections.abc import Mapping
from typing import Any, Literal

from ....llm.data.qwen.schema import QwenChatSchemaHandler
from ..schema import MLLMSchemaHandler
from ..types import MLLMMediaSlot, MLLMSegment

IMAGE_PLACEHOLDER = "<image>"
_MEDIA_MARK = "\x00MEDIA{}\x00"


class QwenVLChatSchemaHandler(MLLMSchemaHandler):
    def __init__(self, processor: Any, *, thinking_mode: bool | None | Literal["non-empty"] = True,
                 image_placeholders: tuple[str, ...] | None = None, image_field: str = "images") -> None:
        """``image_placeholders``: extra strings in message text that stand for the next image (besides
        ``<image>``, the processor's image token and that token wrapped in the vision start / end tokens)."""
        self.processor = processor
        self.image_field = image_field
        self._text = QwenChatSchemaHandler(getattr(processor, "tokenizer", processor), thinking_mode=thinking_mode)
        token = getattr(processor, "image_token", "<|image_pad|>")
        marks = (*(image_placeholders or ()), f"<|vision_start|>{token}<|vision_end|>", IMAGE_PLACEHOLDER, token)
        # longest first, so a wrapped token is taken whole before its inner token could match
        self._placeholder_re = re.compile("|".join(re.escape(m) for m in sorted(set(marks), key=len, reverse=True)))

    def check_row(self, row: Mapping[str, Any]) -> str | None:
        reason = self._text.check_row(row)
        if reason is not None:
            return reason
        for i, im in enumerate(row.get(self.image_field) or []):
            if self._size(row, im, i) is None:
                return "raw.invalid_image_size"
        return None

    def _size(self, row, im, i):
        sizes = row.get("image_sizes")
        if sizes is not None and i < len(sizes):
            return [int(sizes[i][0]), int(sizes[i][1])]
        if isinstance(im, dict) and "height" in im and "width" in im:
            return [int(im["height"]), int(im["width"])]
        return None

    def normalize(self, row):
        reason = self.check_row(row)
        if reason is not None:
            raise ValueError(reason)
        images = row.get(self.image_field) or []
        slots = [MLLMMediaSlot(f"image_{i}", "image", self.image_field, i, {"size": self._size(row, im, i)})
                 for i, im in enumerate(images)]
        counter = iter(range(len(images)))
        msgs = []
        for m in row.get("messages") or row.get("conversations"):
            content = m.get("content", m.get("value"))
            if isinstance(content, list):
                parts = []
                for item in content:
                    if isinstance(item, dict) and item.get("type") in ("image", "image_url"):
                        parts.append(_MEDIA_MARK.format(next(counter)))
                    elif isinstance(item, dict):
                        parts.append(str(item.get("text", "")))
                    else:
                        parts.append(str(item))
                content = "".join(parts)
            content = self._placeholder_re.sub(lambda _: _MEDIA_MARK.format(next(counter)), content)
            msgs.append({**m, "content": content})
        text_segs, meta = self._text.normalize({"messages": msgs})
        segs: list[MLLMSegment] = []
        for seg in text_segs:
            for piece in re.split(r"(\x00MEDIA\d+\x00)", seg.value):
                if not piece:
                    continue
                mm = re.fullmatch(r"\x00MEDIA(\d+)\x00", piece)
                if mm:
                    segs.append(MLLMSegment("image", False, f"image_{int(mm.group(1))}"))
                else:
                    segs.append(MLLMSegment("text", seg.loss, piece))
        return segs, slots, {**meta, "schema": "qwen_vl_chat"}
