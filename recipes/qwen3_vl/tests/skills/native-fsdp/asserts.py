"""Skill asserts: the native flat-buffer FSDP runtime.

Copy to ``recipes/<recipe>/tests/skills/native-fsdp/asserts.py``.  The runtime keeps each unit's
parameters in one contiguous buffer with this rank's slice as the fp32 master, accumulates weight
gradients in fp32 straight from the GEMM epilogues and takes the token-normalisation factor and the clip
coefficient inside its fused AdamW; so a recipe must build the optimizer through ``OptimKit`` (which
returns the flat optimizer for such models) and pass the model itself, not its parameters, to the
rescale.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls


def test_config_structure(config):
    assert config_get(config, "parallel.backend_kwargs.impl", "native") in ("native", "torch")
    r = config_get(config, "parallel.backend_kwargs.reshard_after_forward")
    assert r in (None, True, False), "reshard_after_forward: unset (decide from memory), true or false"


def test_engine_structure(engine_class):
    expect_calls(engine_class, "prepare_optimizer", ["optim_kit.build_optimizer(", "self.model"])
    expect_calls(engine_class, "optimizer_step", ["scale_gradients_", "rescale_gradients("],
                 "the native runtime folds the gradient scale into its update")
    expect_calls(engine_class, "backward_step", ["accumulate_gradients(", "sync=ctx.should_sync"],
                 "gradients are reduced only on the last micro-batch of a step")


def assert_before_train_end(engine):
    if config_get(engine.config, "parallel.backend_kwargs.impl", "native") != "native":
        return
    model = engine.model
    for name in ("scale_gradients_", "grad_shards", "checkpoint_state_dict", "set_requires_gradient_sync"):
        assert hasattr(model, name), f"the native runtime wrapper must provide {name}"
    if config_get(engine.config, "optim.optimizer", "AdamW") == "AdamW":
        assert type(engine.optimizer).__name__ == "FlatAdamW", "AdamW on a native model is the flat fused AdamW"
