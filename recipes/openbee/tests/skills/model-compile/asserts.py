"""Structure asserts of the model-compile skill (reference: recipes/openbee/tests/skills/model-compile/asserts.py).

The engine must route ``model.compile`` config through ``MLLMModelKit.apply_model_compile``, which
compiles with the configured backend / mode (the vision forward stays eager)."""

import inspect
import textwrap

from mvp_engine.kit.mllm import MLLMModelKit


def test_config_structure(config):
    c = config["model"]["compile"] if isinstance(config, dict) else config.model.compile
    get = (lambda k: c[k]) if isinstance(c, dict) else (lambda k: getattr(c, k))
    assert get("enabled") in (True, False)
    assert get("backend") in ("inductor", "aot_eager", "eager")
    assert get("mode") in ("default", "reduce-overhead", "max-autotune", "max-autotune-no-cudagraphs")


def test_engine_structure(engine_class):
    src = "".join(textwrap.dedent(inspect.getsource(k.prepare_model)) for k in engine_class.__mro__
                  if "prepare_model" in k.__dict__)
    for needle in ("m.compile.enabled", "m.compile.backend", "m.compile.mode", "apply_model_compile"):
        assert needle in src, needle
    kit_src = inspect.getsource(MLLMModelKit.apply_model_compile)
    assert "model.compile(backend=backend, mode=mode)" in kit_src
