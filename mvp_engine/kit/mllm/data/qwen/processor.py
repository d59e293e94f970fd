"""Qwen-VL style image processing without the Hugging Face processor files.

* ``smart_resize``: round (H, W) to multiples of ``patch * merge`` while keeping
  the pixel count inside [min_pixels, max_pixels] and the aspect ratio close;
* ``QwenVLImageProcessor``: normalise, repeat the frame ``temporal_patch_size``
  times and cut it into patches in the order Qwen-VL's vision tower expects --
  2x2 merge blocks in raster order, the four patches of a block consecutive,
  each patch flattened as (channel, time, row, col);
* ``QwenVLProcessor``: tokenizer + image processor + the ``<|image_pad|>`` token.

When a real ``transformers`` processor can be loaded it is used instead
(``MLLMDataKit.build_processor``); this class covers offline and synthetic runs.
"""

from __future__ import annotations

import math
from typing import Any, Sequence

import torch

from .....data import SyntheticTokenizer


def smart_resize(height: int, width: int, factor: int = 32, min_pixels: int = 64 * 32 * 32,
                 max_pixels: int = 16384 * 32 * 32) -> tuple[int, int]:
    if max(height, width) / max(1, min(height, width)) > 200:
        raise ValueError(f"aspect ratio of {height}x{width} is too extreme")
    h = max(factor, round(height / factor) * factor)
    w = max(factor, round(width / factor) * factor)
    if h * w > max_pixels:
        s = math.sqrt(height * width / max_pixels)
        h = max(factor, math.floor(height / s / factor) * factor)
        w = max(factor, math.floor(width / s / factor) * factor)
    elif h * w < min_pixels:
        s = math.sqrt(min_pixels / (height * width))
        h = math.ceil(height * s / factor) * factor
        w = math.ceil(width * s / factor) * factor
    return h, w


class QwenVLImageProcessor:
    def __init__(self, patch_size: int = 16, merge_size: int = 2, temporal_patch_size: int = 2,
                 min_pixels: int = 64 * 32 * 32, max_pixels: int = 1024 * 1024,
                 image_mean: Sequence[float] = (0.5, 0.5, 0.5), image_std: Sequence[float] = (0.5, 0.5, 0.5)):
        self.patch_size = patch_size
        self.merge_size = merge_size
        self.temporal_patch_size = temporal_patch_size
        self.size = {"shortest_edge": min_pixels, "longest_edge": max_pixels}
        self.image_mean = torch.tensor(image_mean).view(3, 1, 1)
        self.image_std = torch.tensor(image_std).view(3, 1, 1)

    def patchify(self, img: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """[3, H, W] float -> (patches [gh*gw, 3*tp*p*p], grid_thw [3])."""
        C, H, W = img.shape
        p, m, tp = self.patch_size, self.merge_size, self.temporal_patch_size
        gh, gw = H // p, W // p
        frames = img.unsqueeze(0).expand(tp, C, H, W)
        x = frames.reshape(1, tp, C, gh // m, m, p, gw // m, m, p)
        x = x.permute(0, 3, 6, 4, 7, 2, 1, 5, 8)  # t, bh, bw, mh, mw, c, tp, ph, pw
        return x.reshape(gh * gw, C * tp * p * p), torch.tensor([1, gh, gw])

    def __call__(self, images: Sequence[torch.Tensor], do_resize: bool = False, return_tensors: str = "pt",
                 normalize: bool = True) -> dict[str, torch.Tensor]:
        pix, grids = [], []
        for img in images:
            img = img.float()
            if normalize:
                img = (img - self.image_mean) / self.image_std
            pt, g = self.patchify(img)
            pix.append(pt)
            grids.append(g)
        return {"pixel_values": torch.cat(pix), "image_grid_thw": torch.stack(grids)}


class QwenVLProcessor:
    image_token = "<|image_pad|>"
    video_token = "<|video_pad|>"

    def __init__(self, tokenizer: Any = None, image_processor: QwenVLImageProcessor | None = None) -> None:
        self.tokenizer = tokenizer or SyntheticTokenizer()
        self.image_processor = image_processor or QwenVLImageProcessor()
        self.chat_template = None

    @property
    def min_image_size(self) -> int:
        return int(self.image_processor.size["shortest_edge"])

    @property
    def max_image_size(self) -> int:
        return int(self.image_processor.size["longest_edge"])
