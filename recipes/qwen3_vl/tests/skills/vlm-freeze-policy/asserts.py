"""Skill asserts: freezing the vision tower, the projector or the language model of a VLM.

Copy to ``recipes/<recipe>/tests/skills/vlm-freeze-policy/asserts.py``.  Freezing happens once, on the
bare model and before the data-parallel runtime builds its flat buffers: frozen parameters get no
gradient buffer and no optimizer state there, so the flags cannot change after ``prepare_model``.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls, expect_order

_FLAGS = ("freeze_vit", "freeze_projector", "freeze_llm")
# parameter-name prefixes of each part of the Qwen3-VL model (the kit's defaults)
_PARTS = {
    "freeze_vit": ("model.visual.patch_embed.", "model.visual.blocks.", "model.visual.pos_embed."),
    "freeze_projector": ("model.visual.merger.", "model.visual.deepstack_merger_list."),
    "freeze_llm": ("model.language_model.", "lm_head."),
}


def test_config_structure(config):
    flags = [bool(config_get(config, f"model.{f}", False)) for f in _FLAGS]
    assert not all(flags), "freezing the vision tower, the projector and the LLM leaves nothing to train"


def test_engine_structure(engine_class):
    expect_calls(engine_class, "prepare_model", ["apply_freeze_policy("] + [f"freeze_{p}=" for p in
                                                                              ("vit", "projector", "llm")])
    expect_order(engine_class, "prepare_model", ["apply_freeze_policy(", "parallelize_model("],
                 "freeze before the runtime allocates gradients and optimizer state")


def assert_before_train_end(engine):
    model = engine.unwrapped_model
    for flag, prefixes in _PARTS.items():
        frozen = bool(config_get(engine.config, f"model.{flag}", False))
        for name, p in model.named_parameters():
            if name.startswith(prefixes):
                assert p.requires_grad != frozen, f"{name}: requires_grad must be {not frozen} with {flag}={frozen}"
