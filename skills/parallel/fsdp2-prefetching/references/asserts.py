"""Skill asserts: explicit FSDP2 prefetch edges (torch backend).

Copy to ``recipes/<recipe>/tests/skills/fsdp2-prefetching/asserts.py``.  A model class may define
``APPLY_FSDP2_CUSTOM_PREFETCHING(model)``; the torch backend calls it after ``fully_shard`` so the model
can set ``set_modules_to_forward_prefetch`` / ``set_modules_to_backward_prefetch`` between its blocks.
The native runtime prefetches by itself (one unit ahead) and ignores the hook.
"""

from mvp_engine.testing.skill_checks import config_get


def test_config_structure(config):
    fsdp2 = config_get(config, "parallel.backend_kwargs.fsdp2")
    assert fsdp2 is not None, "parallel.backend_kwargs.fsdp2 must exist"
    assert config_get(fsdp2, "reshard_after_forward") in (True, False)


def check_prefetch_hook(model_class):
    """The hook, when defined, is a callable taking the sharded model (call from a model test)."""
    hook = getattr(model_class, "APPLY_FSDP2_CUSTOM_PREFETCHING", None)
    if hook is None:
        return False
    assert callable(hook), "APPLY_FSDP2_CUSTOM_PREFETCHING must be callable"
    return True


def assert_before_train_end(engine):
    if config_get(engine.config, "parallel.backend_kwargs.impl", "native") != "torch":
        return
    model = engine.unwrapped_model
    if check_prefetch_hook(type(model)):
        blocks = [m for m in model.modules() if hasattr(m, "set_modules_to_forward_prefetch")]
        assert blocks, "the prefetch hook needs fully_shard-ed blocks to link"
