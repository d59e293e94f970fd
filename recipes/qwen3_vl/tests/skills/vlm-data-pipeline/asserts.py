"""Skill asserts: the multimodal data pipeline (MLLMDataKit).

Copy to ``recipes/<recipe>/tests/skills/vlm-data-pipeline/asserts.py``.  The pipeline is declared as one
``MLLMDataSpec`` (source -> sample handlers -> packing -> loader -> rank distribution) and built by the
kit; the engine turns each collated batch into model inputs on the host and copies it once.  The runtime
check verifies the invariant every later stage relies on: the number of image placeholder tokens equals
the number of merged vision patches.
"""

import torch

from mvp_engine.testing.skill_checks import expect_calls, phase_source


def test_engine_structure(engine_class):
    expect_calls(engine_class, "prepare_dataloader", ["build_processor(", "build_dataset(", "build_dataloader("])
    spec_src = phase_source(engine_class, "_data_spec") or phase_source(engine_class, "prepare_dataloader")
    for needle in ("MLLMDataSpec(", "MLLMSampleSpec(", "schema_handler=", "media_handler=", "tokenization_handler=",
                   "build_distribution_spec("):
        assert needle in spec_src, f"the data spec must set {needle}"
    expect_calls(engine_class, "train_pre_step", ["to_device("], "the batch goes to the device once, prepared")


def assert_train_pre_step_end(engine, ctx):
    data = ctx.data
    for key in ("input_ids", "labels", "position_ids", "cu_seq_lens_q"):
        assert key in data, f"prepared batch must carry {key}"
    grid = data.get("image_grid_thw")
    if grid is None or not len(grid):
        return
    model = engine.unwrapped_model
    cfg = model.config
    merge = int(cfg.vision_config.spatial_merge_size)
    patches = int(torch.as_tensor(grid).prod(dim=-1).sum()) // (merge * merge)
    placeholders = int((data["input_ids"] == int(cfg.image_token_id)).sum())
    assert placeholders == patches, f"{placeholders} image tokens for {patches} merged patches"
    assert data["position_ids"].shape[0] == 3, "Qwen3-VL positions are 3-D (t, h, w) M-RoPE ids"
