"""Qwen-VL chat rows -> segments + image slots (reference: mvp_engine/kit/mllm/data/qwen/schema.py:22-332).

Messages may carry content lists with ``{"type": "image", ...}`` items or
``<image>`` placeholders in text; every image becomes an ``MLLMMediaSlot``
(size from ``image_sizes`` / the item's ``height``/``width``) and an image
segment at its position.  User/assistant pairs split into unsupervised prompt
text and supervised response text through the chat template (ChatML when the
tokenizer has none), with the same ``thinking_mode`` rules as the text kit.
"""

from __future__ import annotations

import io
import re
from collections.abc import Mapping
from typing import Any, Literal

from ....llm.data.qwen.schema import QwenChatSchemaHandler
from ..schema import MLLMSchemaHandler
from ..types import MLLMMediaSlot, MLLMSegment

IMAGE_PLACEHOLDER = "<image>"
_MEDIA_MARK = "\x00MEDIA{}\x00"


class _Drop(Exception):
    """A row the handler cannot use; ``reason`` is the guard's drop reason."""

    def __init__(self, reason: str) -> None:
        super().__init__(reason)
        self.reason = reason


def _positive_hw(h: Any, w: Any) -> list[int]:
    try:
        h, w = int(h), int(w)
    except (TypeError, ValueError):
        raise _Drop("raw.invalid_image_size") from None
    if h <= 0 or w <= 0:
        raise _Drop("raw.invalid_image_size")
    return [h, w]


def _hw_of_width_first(size: Any) -> list[int]:
    """[height, width] of a size in the reference's columns: ``{"width", "height"}`` or ``[width, height]``."""
    if isinstance(size, Mapping):
        return _positive_hw(size.get("height"), size.get("width"))
    if isinstance(size, (list, tuple)) and len(size) >= 2:
        return _positive_hw(size[1], size[0])
    raise _Drop("raw.invalid_image_size")


def _probe_hw(image: Any) -> list[int]:
    """[height, width] from the image itself: a tensor's shape, or the header of an encoded image / file."""
    if isinstance(image, Mapping):
        if "seed" in image:  # synthetic image spec without its size
            raise _Drop("raw.invalid_image_size")
        image = image.get("bytes") or image.get("path")
    if hasattr(image, "shape") and len(image.shape) == 3:
        return _positive_hw(image.shape[1], image.shape[2])
    try:
        from PIL import Image
    except ImportError:  # pragma: no cover - PIL ships with the image stack
        raise _Drop("raw.invalid_image_size") from None
    if hasattr(image, "size") and hasattr(image, "mode"):  # already a PIL image
        w, h = image.size
        return _positive_hw(h, w)
    try:
        src = io.BytesIO(image) if isinstance(image, (bytes, bytearray)) else image
        with Image.open(src) as im:  # reads the header only
            w, h = im.size
    except (OSError, TypeError, ValueError, AttributeError):
        raise _Drop("raw.invalid_image_size") from None
    return _positive_hw(h, w)


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
        try:
            self._media(row)
        except _Drop as drop:
            return drop.reason
        return None

    def _media(self, row: Mapping[str, Any]) -> list[tuple[str, int, list[int]]]:
        """(column, index, [height, width]) of every image of ``row``, in placeholder order.

        Accepted layouts: a ``media`` column of ``{"type": "image", "value" | "image": data, "size" |
        "image_size" | "img_size": size}`` entries; or the ``images`` column with sizes from
        ``img_size`` / ``image_size`` (the reference's columns: ``[width, height]`` pairs or
        ``{"width", "height"}`` dicts), ``image_sizes`` (``[height, width]`` pairs), ``height`` / ``width``
        keys of the image item, or, when none is given, the image's own header (read with PIL)."""
        media = row.get("media")
        if media is not None:
            if not isinstance(media, (list, tuple)):
                raise _Drop("raw.invalid_media")
            out = []
            for i, entry in enumerate(media):
                if not isinstance(entry, Mapping):
                    raise _Drop("raw.invalid_media_entry")
                if entry.get("type", "image") != "image":
                    raise _Drop("raw.unsupported_media_type")
                value = entry.get("value", entry.get("image"))
                if value is None:
                    raise _Drop("raw.media_without_value")
                size = entry.get("size") or entry.get("image_size") or entry.get("img_size")
                out.append(("media", i, _hw_of_width_first(size) if size is not None else _probe_hw(value)))
            return out
        images = row.get(self.image_field) or []
        if not isinstance(images, (list, tuple)):
            raise _Drop("raw.invalid_images")
        width_first = row.get("img_size") or row.get("image_size")
        if width_first is not None and len(width_first) != len(images):
            raise _Drop("raw.image_size_count_mismatch")
        hw_sizes = row.get("image_sizes")
        out = []
        for i, im in enumerate(images):
            if width_first is not None:
                hw = _hw_of_width_first(width_first[i])
            elif hw_sizes is not None and i < len(hw_sizes):
                hw = _positive_hw(hw_sizes[i][0], hw_sizes[i][1])
            elif isinstance(im, Mapping) and "height" in im and "width" in im:
                hw = _positive_hw(im["height"], im["width"])
            else:
                hw = _probe_hw(im)
            out.append((self.image_field, i, hw))
        return out

    def normalize(self, row):
        reason = self._text.check_row(row)
        if reason is not None:
            raise ValueError(reason)
        try:
            media = self._media(row)
        except _Drop as drop:
            raise ValueError(drop.reason) from None
        slots = [MLLMMediaSlot(f"image_{i}", "image", column, index, {"size": hw})
                 for i, (column, index, hw) in enumerate(media)]
        counter = iter(range(len(media)))

        def mark(_=None) -> str:
            i = next(counter, None)
            if i is None:
                raise ValueError("raw.more_image_placeholders_than_images")
            return _MEDIA_MARK.format(i)
        msgs = []
        for m in row.get("messages") or row.get("conversations"):
            content = m.get("content", m.get("value"))
            if isinstance(content, list):
                parts = []
                for item in content:
                    if isinstance(item, dict) and item.get("type") in ("image", "image_url"):
                        parts.append(mark())
                    elif isinstance(item, dict):
                        parts.append(str(item.get("text", "")))
                    else:
                        parts.append(str(item))
                content = "".join(parts)
            content = self._placeholder_re.sub(mark, content)
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
