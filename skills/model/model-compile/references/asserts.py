"""Skill asserts: torch.compile wiring through the model kit.

Copy to ``recipes/<recipe>/tests/skills/model-compile/asserts.py``.  Compilation is optional and never
the hot path of this engine (its kernels are opaque to the compiler); the kit compiles the language
model and leaves a vision tower eager, because image shapes change from batch to batch.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls, expect_order

_BACKENDS = ("inductor", "aot_eager", "eager")
_MODES = ("default", "reduce-overhead", "max-autotune", "max-autotune-no-cudagraphs")


def test_config_structure(config):
    c = config_get(config, "model.compile")
    assert c is not None, "model.compile must exist (enabled / backend / mode)"
    assert config_get(c, "enabled") in (True, False)
    assert config_get(c, "backend") in _BACKENDS, config_get(c, "backend")
    assert config_get(c, "mode") in _MODES, config_get(c, "mode")


def test_engine_structure(engine_class):
    expect_calls(engine_class, "prepare_model",
                 ["compile.enabled", "apply_model_compile(", "compile.backend", "compile.mode"])
    expect_order(engine_class, "prepare_model", ["apply_model_compile(", "parallelize_model("],
                 "compile the bare model; the data-parallel runtime wraps the compiled modules")
