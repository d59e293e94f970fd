"""Row -> training sample for the minimal VLM recipe (reference: recipes/minimal_vlm/dataset/preprocess.py:30-534).

Same behaviour as the reference's hand-rolled preprocessing, expressed with the multimodal kit's
handlers: the chat (or synthetic token) schema gives text segments and image slots; images are
smart-resized to multiples of 32 px within the processor's pixel bounds and patchified; every
image placeholder expands to ``t*h*w/4`` image tokens; only assistant text is supervised (prompt,
template and image tokens get label -100); a sample whose truncation to ``max_length`` would cut
image tokens is dropped instead of corrupting the image/text alignment.
"""

from __future__ import annotations

import io
from pathlib import Path
from typing import Any, Optional, Union

import torch

from mvp_engine.kit.mllm import MLLMSample, MLLMSampleSpec, QwenVLChatSchemaHandler, QwenVLMediaHandler
from mvp_engine.kit.mllm import QwenVLTokenizationHandler
from mvp_engine.kit.mllm.data import SyntheticVLSchemaHandler
from mvp_engine.kit.mllm.data.qwen.media import QwenImageHandler, read_image
from mvp_engine.kit.mllm.data.types import MLLMMediaSlot

IMAGE_PLACEHOLDER = "<image>"


def build_sample_spec(processor: Any, max_length: int, synthetic: bool, *, image_placeholder: str = IMAGE_PLACEHOLDER,
                      ignore_index: int = -100) -> MLLMSampleSpec:
    schema = SyntheticVLSchemaHandler() if synthetic else QwenVLChatSchemaHandler(
        processor=processor, image_placeholders=(image_placeholder,))
    return MLLMSampleSpec(schema_handler=schema, media_handler=QwenVLMediaHandler(processor=processor),
                          tokenization_handler=QwenVLTokenizationHandler(tokenizer=processor.tokenizer,
                                                                         max_seq_len=int(max_length),
                                                                         ignore_index=int(ignore_index)))


def process_image(image: Any, *, image_root: Optional[Path] = None):
    """One image of a row (path, bytes, ``{"bytes"|"path"}`` record or PIL image) as an RGB PIL image;
    relative paths resolve against ``image_root``."""
    from PIL import Image

    if isinstance(image, dict):
        data = image.get("bytes")
        if isinstance(data, (bytes, bytearray, memoryview)):
            return process_image(bytes(data), image_root=image_root)
        if isinstance(image.get("path"), str) and image["path"]:
            return process_image(image["path"], image_root=image_root)
        raise ValueError("contains an invalid image record.")
    if isinstance(image, Image.Image):
        return image.convert("RGB").copy()
    if isinstance(image, (bytes, bytearray)):
        with Image.open(io.BytesIO(bytes(image))) as img:
            return img.convert("RGB")
    if not isinstance(image, str) or not image:
        raise ValueError(f"contains an invalid image value: {image!r}")
    path = Path(image).expanduser()
    if not path.is_absolute() and image_root is not None:
        path = Path(image_root) / path
    if not path.is_file():
        raise FileNotFoundError(f"references missing image: {path.resolve()}")
    with Image.open(path) as img:
        return img.convert("RGB").copy()


def convert_images_to_pixel_values(sample: Union[dict, list], *, processor: Any) -> Union[dict, list]:
    """Replace a row's ``images`` (resized to its ``adjusted_image_size`` entries, or to the processor's
    smart-resize of each image) by ``pixel_values`` / ``image_grid_thw``; lists are converted element-wise."""
    if isinstance(sample, list):
        return [convert_images_to_pixel_values(s, processor=processor) for s in sample]
    images = sample.pop("images", None) or []
    sizes = sample.pop("adjusted_image_size", None) or []
    if not images:
        return sample
    import torch.nn.functional as F

    handler = QwenImageHandler()
    tensors = []
    for i, image in enumerate(images):
        pil = process_image(image)
        if i < len(sizes):  # the size the row was tokenised for (already a multiple of patch x merge)
            h, w = int(sizes[i][0]), int(sizes[i][1])
        else:
            slot = MLLMMediaSlot(f"image_{i}", "image", "images", i, {"size": [pil.height, pil.width]})
            h, w = handler.adjusted_size(slot, processor=processor)
        t = read_image(pil)
        if tuple(t.shape[1:]) != (h, w):
            t = F.interpolate(t.unsqueeze(0), size=(h, w), mode="bicubic", align_corners=False)[0]
        tensors.append(t)
    out = processor.image_processor(images=tensors, do_resize=False, return_tensors="pt")
    sample["pixel_values"], sample["image_grid_thw"] = out["pixel_values"], out["image_grid_thw"]
    return sample


def process_sample(sample: dict[str, Any], *, processor: Any = None, max_length: Optional[int] = None,
                   image_placeholder: str = IMAGE_PLACEHOLDER, ignore_index: int = -100,
                   spec: Optional[MLLMSampleSpec] = None) -> Optional[dict[str, Any]]:
    """One row -> {input_ids, attention_mask, labels[, pixel_values, image_grid_thw]} or None (dropped).

    Pass the reference's arguments (``processor``, ``max_length``, ``image_placeholder``, ``ignore_index``) or
    a prepared ``spec`` (what the recipe's dataset does, building it once)."""
    if spec is None:
        if processor is None or max_length is None:
            raise ValueError("process_sample needs processor and max_length, or a sample spec")
        spec = build_sample_spec(processor, int(max_length), synthetic=False, image_placeholder=image_placeholder,
                                 ignore_index=ignore_index)
    row = sample
    sample = MLLMSample.from_row(row, sample_spec=spec).load_media()
    if not sample.input_ids:
        return None
    out = {"input_ids": torch.tensor(sample.input_ids, dtype=torch.long),
           "attention_mask": torch.tensor(sample.attention_mask, dtype=torch.long),
           "labels": torch.tensor(sample.labels, dtype=torch.long)}
    media = sample.media or {}
    for key in ("pixel_values", "image_grid_thw"):
        if media.get(key) is not None:
            out[key] = media[key]
    return out
