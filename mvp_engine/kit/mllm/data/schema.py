"""Row -> (segments, media slots, metadata) normalisation (reference: mvp_engine/kit/mllm/data/schema.py:20-39)."""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any

from .types import MLLMMediaSlot, MLLMSegment


class MLLMSchemaHandler:
    def check_row(self, row: Mapping[str, Any]) -> str | None:
        return None

    def normalize(self, row: Mapping[str, Any]) -> tuple[list[MLLMSegment], list[MLLMMediaSlot], dict[str, Any]]:
        raise NotImplementedError


class SyntheticVLSchemaHandler(MLLMSchemaHandler):
    """Rows of the ``synthetic_mm`` source: text token segments interleaved with images.

    The last ``loss_fraction`` of every text segment is supervised (answer
    text), the rest is prompt; image placeholders are never supervised.
    """

    def check_row(self, row: Mapping[str, Any]) -> str | None:
        if not isinstance(row.get("text_segments"), list):
            return "raw.invalid_text_segments"
        imgs = row.get("images") or []
        if len(row["text_segments"]) != len(imgs) + 1:
            return "raw.segment_image_mismatch"
        return None

    def normalize(self, row):
        frac = float(row.get("loss_fraction", 0.3))
        segs: list[MLLMSegment] = []
        slots: list[MLLMMediaSlot] = []
        images = row.get("images") or []
        for i, toks in enumerate(row["text_segments"]):
            cut = int(round(len(toks) * (1.0 - frac)))
            if cut:
                segs.append(MLLMSegment("tokens", False, list(toks[:cut])))
            if len(toks) - cut:
                segs.append(MLLMSegment("tokens", True, list(toks[cut:])))
            if i < len(images):
                im = images[i]
                mid = f"image_{i}"
                slots.append(MLLMMediaSlot(mid, "image", "images", i, {"size": [int(im["height"]), int(im["width"])]}))
                segs.append(MLLMSegment("image", False, mid))
        return segs, slots, {"schema": "synthetic_vl"}
