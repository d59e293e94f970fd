"""Multimodal data kit on CPU: processor geometry, schema, packing, collation, guards."""

import pytest
import torch

from mvp_engine.kit.mllm import (MLLMDataKit, MLLMDataSpec, MLLMLoaderSpec, MLLMPackingSpec, MLLMSampleSpec,
                                 MLLMSourceSpec, MLLMTextOnlyBatchGuard, QwenImageHandler, QwenVLMediaHandler,
                                 QwenVLTokenizationHandler)
from mvp_engine.kit.mllm.data import SyntheticVLSchemaHandler, smart_resize


def test_smart_resize_bounds():
    h, w = smart_resize(1000, 700, factor=32, min_pixels=64 * 1024, max_pixels=1024 * 1024)
    assert h % 32 == 0 and w % 32 == 0 and h * w <= 1024 * 1024
    assert smart_resize(448, 448, factor=32, min_pixels=1, max_pixels=1 << 30) == (448, 448)


def _spec(max_len=4096):
    kit = MLLMDataKit()
    proc = kit.build_processor("synthetic", image_max_pixels=1344 * 1344)
    tok = proc.tokenizer
    sample = MLLMSampleSpec(SyntheticVLSchemaHandler(), QwenVLMediaHandler(proc),
                            QwenVLTokenizationHandler(tok, max_seq_len=max_len))
    src = MLLMSourceSpec("synthetic://mm?min_px=64&max_px=256&num_rows=12&min_text=20&max_text=100",
                         dataset_source="synthetic_mm", resample=False)
    return kit, proc, MLLMDataSpec(src, sample, MLLMPackingSpec(max_len, buffer_size=4, open_pack_limit=2),
                                   MLLMLoaderSpec(batch_size=1))


def test_pipeline_image_tokens_match_features():
    kit, proc, spec = _spec()
    items = list(kit.build_dataset(spec))
    assert items
    image_id = proc.tokenizer.convert_tokens_to_ids("<|image_pad|>")
    for it in items:
        n_tok = int((it["input_ids"] == image_id).sum())
        assert n_tok == int(it["image_grid_thw"].prod(-1).sum()) // 4
        assert it["pixel_values"].shape == (int(it["image_grid_thw"].prod(-1).sum()), 3 * 2 * 16 * 16)
        assert it["input_ids"].numel() <= 4096
        seg = it["pack_segment_ids"]
        assert int(seg.max()) == it["source_sample_num"]


def test_collate_and_text_only_guard():
    kit, proc, spec = _spec()
    loader = kit.build_dataloader(kit.build_dataset(spec), spec)
    b = next(iter(loader))
    assert b["effective_tokens"] > 0 and "pixel_values" in b
    dummy = QwenImageHandler().build_dummy_inputs(proc)
    guard = MLLMTextOnlyBatchGuard(dummy_inputs=dummy, media_keys=("pixel_values", "image_grid_thw"),
                                   pad_token_id=proc.tokenizer.pad_token_id)
    text_only = {k: v for k, v in b.items() if k not in ("pixel_values", "image_grid_thw")}
    out = guard(text_only)
    assert out["pixel_values"].shape[0] == 4 and out["input_ids"].shape[1] >= b["input_ids"].shape[1]
    assert int(out["pack_segment_ids"].max()) == int(b["pack_segment_ids"].max()) + 1


def test_chat_row_through_the_handler_interfaces():
    """The handler contract step by step (schema -> media render -> tokenise, as the reference defines
    it): every image placeholder form in message text takes the next image slot, media segments render to
    unsupervised placeholder tokens, and MLLMSample accepts the handlers directly."""
    from mvp_engine.kit.mllm import MLLMSample, QwenVLChatSchemaHandler
    from mvp_engine.kit.mllm.data.types import MLLMSegment

    proc = MLLMDataKit().build_processor("synthetic", image_max_pixels=256 * 256)
    schema = QwenVLChatSchemaHandler(proc, thinking_mode=None, image_placeholders=("[IMG]",))
    media = QwenVLMediaHandler(proc)
    tok = QwenVLTokenizationHandler(proc.tokenizer, max_seq_len=4096)
    row = {"messages": [{"role": "user", "content": "<image> and [IMG]: compare"},
                        {"role": "assistant", "content": "the first is larger"}],
           "images": [{"height": 64, "width": 64}, {"height": 128, "width": 96}]}
    segs, slots, _ = schema.normalize(row)
    assert [s.value for s in segs if s.type == "image"] == ["image_0", "image_1"] and len(slots) == 2
    rendered = media.render(segs, slots)
    assert all(isinstance(s, MLLMSegment) for s in rendered)
    assert all(s.type == "image" and not s.loss and "<|image_pad|>" in s.value for s in rendered if s.type == "image")
    ids, labels, mask = tok.tokenize(rendered)
    image_id = proc.tokenizer.convert_tokens_to_ids("<|image_pad|>")
    pad_positions = [i for i, t in enumerate(ids) if t == image_id]
    assert pad_positions and all(labels[i] == -100 for i in pad_positions) and len(mask) == len(ids)
    assert any(lab != -100 for lab in labels)  # the assistant reply is supervised
    sample = MLLMSample(row, schema_handler=schema, media_handler=media, tokenization_handler=tok)
    assert sample.input_ids == ids and sample.labels == labels


def _png(w, h, colour=(200, 30, 30)):
    import io

    from PIL import Image

    buf = io.BytesIO()
    Image.new("RGB", (w, h), colour).save(buf, format="PNG")
    return buf.getvalue()


def test_reference_row_layouts_give_the_same_slots(tmp_path):
    """Rows in the reference's layouts -- ``img_size`` / ``image_size`` as [width, height] pairs or dicts,
    or a ``media`` column of {type, value, size} entries -- and rows with no size at all (read from the
    image header) give image slots of the right [height, width], and the media handler loads their pixels."""
    from mvp_engine.kit.mllm import QwenVLChatSchemaHandler

    proc = MLLMDataKit().build_processor("synthetic", image_max_pixels=256 * 256)
    schema = QwenVLChatSchemaHandler(proc, thinking_mode=None)
    media = QwenVLMediaHandler(proc)
    png = _png(96, 64)  # width 96, height 64
    (tmp_path / "i.png").write_bytes(png)
    msgs = [{"role": "user", "content": "<image> what colour?"}, {"role": "assistant", "content": "red"}]
    rows = [
        {"messages": msgs, "images": [png], "img_size": [[96, 64]]},
        {"messages": msgs, "images": [png], "image_size": [{"width": 96, "height": 64}]},
        {"messages": msgs, "images": [{"bytes": png}], "image_sizes": [[64, 96]]},
        {"messages": msgs, "media": [{"type": "image", "value": png, "size": [96, 64]}]},
        {"messages": msgs, "media": [{"image": str(tmp_path / "i.png"), "img_size": {"width": 96, "height": 64}}]},
        {"messages": msgs, "images": [png]},  # no size column: the PNG header gives it
        {"messages": msgs, "images": [str(tmp_path / "i.png")]},
    ]
    grids = []
    for row in rows:
        assert schema.check_row(row) is None, row
        segs, slots, _ = schema.normalize(row)
        assert [s.metadata["size"] for s in slots] == [[64, 96]]
        values = [media._slot_value(row, slot) for slot in slots]
        assert all(isinstance(v, (bytes, str, dict)) for v in values)
        loaded = media.handlers["image"].load(slots, values, processor=proc)
        grids.append(loaded["image_grid_thw"].tolist())
        assert loaded["pixel_values"].shape[0] == int(loaded["image_grid_thw"].prod())
    assert all(g == grids[0] for g in grids)


def test_unusable_media_rows_are_dropped_with_a_reason():
    from mvp_engine.kit.mllm import QwenVLChatSchemaHandler

    proc = MLLMDataKit().build_processor("synthetic", image_max_pixels=256 * 256)
    schema = QwenVLChatSchemaHandler(proc, thinking_mode=None)
    msgs = [{"role": "user", "content": "<image> hi"}, {"role": "assistant", "content": "yo"}]
    png = _png(32, 32)
    cases = {
        "raw.image_size_count_mismatch": {"images": [png], "img_size": [[32, 32], [32, 32]]},
        "raw.invalid_image_size": {"images": [b"not an image"]},
        "raw.unsupported_media_type": {"media": [{"type": "video", "value": png, "size": [32, 32]}]},
        "raw.media_without_value": {"media": [{"type": "image", "size": [32, 32]}]},
        "raw.invalid_media": {"media": "x.png"},
    }
    for reason, extra in cases.items():
        assert schema.check_row({"messages": msgs, **extra}) == reason
    with pytest.raises(ValueError, match="more_image_placeholders"):
        schema.normalize({"messages": [{"role": "user", "content": "<image><image>"},
                                       {"role": "assistant", "content": "a"}], "images": [png]})
