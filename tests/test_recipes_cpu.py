"""Recipe-level tests on CPU: config validation, Qwen3-VL packed positions, engine steps (gloo)."""

from pathlib import Path
from types import SimpleNamespace

import pytest
import torch
import yaml

ROOT = Path(__file__).resolve().parent.parent


def _vl_cfg():
    return SimpleNamespace(image_token_id=9, vision_start_token_id=8, video_token_id=7,
                           vision_config=SimpleNamespace(spatial_merge_size=2))


def test_qwen3_vl_packed_positions_hand_example():
    from recipes.qwen3_vl.model.packing import build_qwen3_vl_packed_position_ids

    # seg 1: a b <vs> img*4 <ve> c   (image grid t=1, h=4, w=4 -> 2x2 merged tokens);  seg 2: d e;  pad
    ids = torch.tensor([[1, 2, 8, 9, 9, 9, 9, 6, 3, 4, 5, 0]])
    seg = torch.tensor([[1, 1, 1, 1, 1, 1, 1, 1, 1, 2, 2, 0]])
    pos = build_qwen3_vl_packed_position_ids(input_ids=ids, pack_segment_ids=seg,
                                             image_grid_thw=torch.tensor([[1, 4, 4]]), model_config=_vl_cfg())
    t, h, w = pos[:, 0].tolist()
    assert t == [0, 1, 2, 3, 3, 3, 3, 5, 6, 7, 8, 1]
    assert h == [0, 1, 2, 3, 3, 4, 4, 5, 6, 7, 8, 1]
    assert w == [0, 1, 2, 3, 4, 3, 4, 5, 6, 7, 8, 1]


def test_qwen3_vl_positions_reject_mismatched_grids():
    from recipes.qwen3_vl.model.packing import build_qwen3_vl_packed_position_ids

    ids = torch.tensor([[8, 9, 9, 9, 9, 1]])
    seg = torch.ones_like(ids)
    with pytest.raises(ValueError):
        build_qwen3_vl_packed_position_ids(input_ids=ids, pack_segment_ids=seg, image_grid_thw=None,
                                           model_config=_vl_cfg())
    with pytest.raises(ValueError):
        build_qwen3_vl_packed_position_ids(input_ids=ids, pack_segment_ids=seg,
                                           image_grid_thw=torch.tensor([[1, 4, 4], [1, 4, 4]]),
                                           model_config=_vl_cfg())


@pytest.mark.parametrize("recipe,schema_mod,cls", [
    ("qwen3", "recipes.qwen3.configs.schema", "Qwen3Config"),
    ("qwen3_vl", "recipes.qwen3_vl.configs.schema", "Qwen3VLConfig"),
])
def test_recipe_configs_validate(recipe, schema_mod, cls):
    import importlib

    from mvp_engine.config.loader import deep_merge, load_yaml

    C = getattr(importlib.import_module(schema_mod), cls)
    default = load_yaml(ROOT / "mvp_engine" / "config" / "default.yaml")
    paths = sorted((ROOT / "recipes" / recipe / "configs").glob("*.yaml"))
    assert paths
    for p in paths:
        cfg = C.model_validate(deep_merge(default, yaml.safe_load(p.read_text())))
        assert cfg.engine


def _run_vl(rank, world, port, steps):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = ROOT / "recipes" / "qwen3_vl"
    import_recipe_modules(root)
    import tempfile

    cfg = load_smoke_test_config(root, "synthetic_tiny", output_dir=Path(tempfile.mkdtemp()),
                                 config_overrides=(f"loop.total_steps={steps}", "checkpoint.interval=1000000",
                                                   f"optim.global_batch_size={2 * world}"))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    eng.train()
    return eng.last_logs


def test_qwen3_vl_engine_trains_on_cpu_two_ranks():
    from mvp_engine.testing.utils import spawn_workers

    logs = spawn_workers(_run_vl, 2, 2, timeout=600)
    for lg in logs:
        assert torch.isfinite(torch.tensor(lg["train/loss"]))
        assert 5.0 < lg["train/loss"] < 13.0
    assert logs[0]["train/loss"] == pytest.approx(logs[1]["train/loss"])
    assert logs[0]["tokens/total"] == logs[1]["tokens/total"]


def _run_vit(rank, world, port, steps, global_batch, impl):
    import tempfile

    import torch.distributed as dist

    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = ROOT / "recipes" / "vit_classification"
    import_recipe_modules(root)
    cfg = load_smoke_test_config(root, "tiny_cpu_fp32", output_dir=Path(tempfile.mkdtemp()),
                                 config_overrides=(f"loop.total_steps={steps}", "checkpoint.interval=1000000",
                                                   f"data.batch_size={global_batch // world}",
                                                   f"parallel.backend_kwargs.impl={impl}"))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    losses = []
    post = eng.train_post_step

    def record(ctx):
        post(ctx)
        l = torch.tensor([eng.last_logs["train/loss"]], dtype=torch.float64)
        if dist.is_initialized() and world > 1:
            dist.all_reduce(l)
            l /= world
        losses.append(float(l))

    eng.train_post_step = record
    eng.train()
    return losses


@pytest.mark.parametrize("impl", ["native", "torch"])
def test_vit_tiny_fsdp_world2_matches_single_process(impl):
    """ViT-Tiny/16 (192 hidden, 3 heads, MLP 768, 12 layers, 1000 classes), fp32, gloo FSDP over 2 ranks with
    per-rank batch 8, AdamW lr 1e-3, 20 steps: the loss curve equals the single-process run with batch 16."""
    from mvp_engine.testing.utils import spawn_workers

    single = spawn_workers(_run_vit, 1, 20, 16, impl, timeout=900)[0]
    multi = spawn_workers(_run_vit, 2, 20, 16, impl, timeout=900)
    assert len(single) == 20 and multi[0] == multi[1]
    for a, b in zip(single, multi[0]):
        assert abs(a - b) <= 1e-4 * max(1.0, abs(a)), (single, multi[0])


def _run_recipe(rank, world, port, recipe, config, overrides):
    import tempfile

    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = ROOT / "recipes" / recipe
    import_recipe_modules(root)
    cfg = load_smoke_test_config(root, config, output_dir=Path(tempfile.mkdtemp()),
                                 config_overrides=("checkpoint.interval=1000000",) + tuple(overrides))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    eng.before_train()
    m = eng.unwrapped_model

    def snapshot():
        if hasattr(eng.model, "checkpoint_state_dict"):  # native runtime: parameters live in flat buffers
            return {n: t.detach().float().clone() for n, t in eng.model.checkpoint_state_dict(full=True).items()}
        return {n: p.detach().float().clone() for n, p in m.named_parameters()}

    before = snapshot()
    eng.do_train()
    after = snapshot()
    changed = sorted(n for n in before if not torch.equal(before[n], after[n]))
    out = {"logs": eng.last_logs, "changed": changed, "names": sorted(before)}
    if recipe == "magic_transformer":
        out["generated"] = m.generate(torch.zeros(1, 4, dtype=torch.long), max_new_tokens=3).shape
    return out


def test_openbee_stage1_trains_only_the_merger():
    from mvp_engine.testing.utils import spawn_workers

    r = spawn_workers(_run_recipe, 1, "openbee", "synthetic_tiny", ("loop.total_steps=2",), timeout=600)[0]
    assert r["changed"], "nothing trained"
    for n in r["changed"]:
        assert n.startswith(("model.visual.merger.", "model.visual.deepstack_merger_list.")), n
    assert any(n.startswith("model.language_model.") for n in r["names"])


def test_minimal_vlm_trains_language_model_only():
    from mvp_engine.testing.utils import spawn_workers

    r = spawn_workers(_run_recipe, 1, "minimal_vlm", "synthetic_tiny", ("loop.total_steps=2",), timeout=600)[0]
    assert 5.0 < r["logs"]["train/loss"] < 13.0
    assert r["changed"] and not any(n.startswith("model.visual.") for n in r["changed"])


def test_magic_transformer_trains_and_generates():
    from mvp_engine.testing.utils import spawn_workers

    r = spawn_workers(_run_recipe, 1, "magic_transformer", "train", ("loop.total_steps=3", "log.interval=1"),
                      timeout=600)[0]
    assert 5.0 < r["logs"]["train/loss"] < 8.0
    assert "embed.weight" in r["changed"] and tuple(r["generated"]) == (1, 7)


def test_minimal_vlm_preprocessing_entry_points(tmp_path):
    """The recipe's row preprocessing with the reference's arguments: image decoding from bytes / path /
    record, pixel conversion, and a chat row with an ``<image>`` placeholder -> supervised-reply tokens
    plus as many image tokens as merged patches."""
    import io

    from PIL import Image

    from mvp_engine.kit.mllm import MLLMDataKit
    from recipes.minimal_vlm.dataset.preprocess import (convert_images_to_pixel_values, process_image,
                                                        process_sample)

    img = Image.new("RGB", (40, 30), (200, 10, 10))
    buf = io.BytesIO()
    img.save(buf, format="PNG")
    png = buf.getvalue()
    (tmp_path / "a.png").write_bytes(png)
    for src in (png, {"bytes": png}, {"path": "a.png"}, img):
        out = process_image(src, image_root=tmp_path)
        assert out.size == (40, 30) and out.mode == "RGB"
    with pytest.raises(FileNotFoundError):
        process_image("missing.png", image_root=tmp_path)

    proc = MLLMDataKit().build_processor("synthetic", image_max_pixels=256 * 256)
    conv = convert_images_to_pixel_values({"images": [png], "adjusted_image_size": [[64, 64]]}, processor=proc)
    assert conv["image_grid_thw"].tolist() == [[1, 4, 4]] and conv["pixel_values"].shape[0] == 16

    row = {"messages": [{"role": "user", "content": "<image> what colour?"},
                        {"role": "assistant", "content": "red"}],
           "images": [{"bytes": png}], "image_sizes": [[64, 64]]}
    s = process_sample(row, processor=proc, max_length=512)
    image_id = proc.tokenizer.convert_tokens_to_ids("<|image_pad|>")
    n_img = int((s["input_ids"] == image_id).sum())
    assert n_img == int(s["image_grid_thw"].prod(-1).sum()) // 4 > 0  # smart-resized within the pixel bounds
    assert int((s["labels"] != -100).sum()) > 0 and bool((s["labels"][s["input_ids"] == image_id] == -100).all())
