"""Qwen-VL image media handler (reference: mvp_engine/kit/mllm/data/qwen/media.py:28-306).

Render: ``<|vision_start|>`` + ``<|image_pad|>`` x N + ``<|vision_end|>`` with
N = (H'/patch)(W'/patch)/merge^2 for the smart-resized size H' x W'.
Load: image -> resize -> normalise -> patches (``pixel_values``) and
``image_grid_thw``.  Synthetic images are dicts ``{height, width, seed}``
whose pixels are drawn N(0, 1) (already "normalised", so no further scaling).
Unreadable media turn the sample into the empty-sample sentinel, which the
guards drop.
"""

from __future__ import annotations

import io
from typing import Any

import torch
import torch.nn.functional as F

from .....utils.log import simple_info
from ..media import MLLMMediaHandler, MLLMMediaTypeHandler, RenderedMedia, empty_model_sample
from ..types import MLLMMediaSlot
from .processor import smart_resize

VISION_START_TOKEN = "<|vision_start|>"
VISION_END_TOKEN = "<|vision_end|>"
DEFAULT_IMAGE_TOKEN = "<|image_pad|>"


def read_image(image: Any) -> torch.Tensor:
    """-> float [3, H, W] in [0, 1] (or N(0,1) for synthetic specs)."""
    if isinstance(image, dict) and "seed" in image and "height" in image:
        g = torch.Generator().manual_seed(int(image["seed"]))
        return torch.randn(3, int(image["height"]), int(image["width"]), generator=g)
    if isinstance(image, torch.Tensor):
        return image.float()
    from PIL import Image  # optional dependency for real images

    if isinstance(image, dict):
        image = image.get("bytes") or image.get("path")
    if isinstance(image, (bytes, bytearray)):
        img = Image.open(io.BytesIO(image))
    elif isinstance(image, str):
        img = Image.open(image)
    else:
        img = image
    import numpy as np

    arr = np.asarray(img.convert("RGB"), dtype=np.float32) / 255.0
    return torch.from_numpy(arr).permute(2, 0, 1).contiguous()


class QwenImageHandler(MLLMMediaTypeHandler):
    media_type = "image"
    DUMMY_IMAGE_PIXELS = 32 * 32
    OUTPUT_TENSOR_KEYS = ("pixel_values", "image_grid_thw")

    def default_token(self, processor: Any) -> str:
        tok = getattr(processor, "image_token", DEFAULT_IMAGE_TOKEN)
        if not isinstance(tok, str) or not tok:
            raise ValueError("Processor must expose a valid image token.")
        return tok

    @staticmethod
    def _geometry(processor: Any) -> tuple[int, int, int, int]:
        ip = getattr(processor, "image_processor", processor)
        size = getattr(ip, "size", {}) or {}
        mn = getattr(processor, "min_image_size", None) or size.get("shortest_edge")
        mx = getattr(processor, "max_image_size", None) or size.get("longest_edge")
        return int(ip.patch_size), int(ip.merge_size), int(mn), int(mx)

    def adjusted_size(self, slot: MLLMMediaSlot, *, processor: Any) -> tuple[int, int]:
        p, m, mn, mx = self._geometry(processor)
        h, w = slot.metadata.get("size") or (slot.metadata.get("height"), slot.metadata.get("width"))
        return smart_resize(int(h), int(w), factor=p * m, min_pixels=mn, max_pixels=mx)

    def render(self, slot: MLLMMediaSlot, *, processor: Any, tokenizer: Any) -> RenderedMedia:
        p, m, _, _ = self._geometry(processor)
        h, w = self.adjusted_size(slot, processor=processor)
        n = (h // p) * (w // p) // (m * m)
        return RenderedMedia(slot.media_id, self.media_type,
                             f"{VISION_START_TOKEN}{self.default_token(processor) * n}{VISION_END_TOKEN}")

    def load(self, slots: list[MLLMMediaSlot], values: list[Any], *, processor: Any) -> dict[str, Any]:
        if not values:
            return {}
        try:
            imgs = []
            synthetic = True
            for slot, v in zip(slots, values):
                img = read_image(v)
                synthetic = synthetic and isinstance(v, dict) and "seed" in v
                h, w = self.adjusted_size(slot, processor=processor)
                if img.shape[1:] != (h, w):
                    img = F.interpolate(img.unsqueeze(0), size=(h, w), mode="bicubic", align_corners=False)[0]
                imgs.append(img)
            out = processor.image_processor(images=imgs, do_resize=False, return_tensors="pt",
                                            **({"normalize": False} if synthetic else {}))
        except FileNotFoundError as exc:
            simple_info(f"dropping sample with missing image media: {exc}", level="warning")
            return empty_model_sample()
        except (OSError, ValueError) as exc:
            simple_info(f"dropping sample with unreadable media: {exc}", level="warning")
            return empty_model_sample()
        return {"pixel_values": out["pixel_values"], "image_grid_thw": out["image_grid_thw"]}

    def build_dummy_inputs(self, processor: Any) -> dict[str, torch.Tensor]:
        """Smallest valid image suffix (32x32 -> 1 merged token) for text-only batches."""
        tok = processor.tokenizer
        slot = MLLMMediaSlot("dummy", "image", "images", 0, {"size": [32, 32]})
        text = self.render(slot, processor=processor, tokenizer=tok).text
        ids = _encode(tok, text)
        out = processor.image_processor(images=[torch.zeros(3, 32, 32)], do_resize=False, return_tensors="pt")
        return {"input_ids": torch.tensor(ids, dtype=torch.long), "attention_mask": torch.ones(len(ids), dtype=torch.long),
                "pixel_values": out["pixel_values"], "image_grid_thw": out["image_grid_thw"]}


def _encode(tok: Any, text: str) -> list[int]:
    enc = tok(text, add_special_tokens=False)
    return list(enc["input_ids"] if isinstance(enc, dict) or hasattr(enc, "keys") else enc)


class QwenVLMediaHandler(MLLMMediaHandler):
    def __init__(self, processor: Any, handlers: dict[str, MLLMMediaTypeHandler] | None = None) -> None:
        super().__init__(processor=processor, handlers=handlers or {"image": QwenImageHandler()})
