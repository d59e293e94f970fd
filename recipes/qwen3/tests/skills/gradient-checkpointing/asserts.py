"""Skill asserts: activation checkpointing through the model kit.

Copy to ``recipes/<recipe>/tests/skills/gradient-checkpointing/asserts.py``.  Recomputation is switched
on before the model is handed to the data-parallel runtime (whose units are the decoder layers), and
``num_layers`` limits it to the first layers so the rest keep their activations.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls, expect_order


def test_config_structure(config):
    gc = config_get(config, "model.gradient_checkpointing")
    assert gc is not None, "model.gradient_checkpointing must exist (enabled / use_reentrant / num_layers)"
    assert config_get(gc, "enabled") in (True, False)
    assert config_get(gc, "use_reentrant") in (True, False)
    n = config_get(gc, "num_layers")
    assert n is None or int(n) >= 0, "num_layers: None (every layer) or a count"


def test_engine_structure(engine_class):
    expect_calls(engine_class, "prepare_model",
                 ["gradient_checkpointing.enabled", "apply_gradient_checkpointing(", "use_reentrant", "num_layers"])
    expect_order(engine_class, "prepare_model",
                 ["apply_freeze_policy(", "apply_gradient_checkpointing(", "parallelize_model("],
                 "wrap for recomputation after freezing and before data-parallel wrapping")


def _recomputes(model):
    for m in model.modules():
        if getattr(m, "gradient_checkpointing", False) or hasattr(m, "_checkpoint_wrapped_module"):
            return True
    return False


def assert_before_train_end(engine):
    enabled = bool(config_get(engine.config, "model.gradient_checkpointing.enabled", False))
    assert _recomputes(engine.unwrapped_model) == enabled, (
        "the built model must recompute activations exactly when model.gradient_checkpointing.enabled is set")
