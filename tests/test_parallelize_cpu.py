"""Runtime selection of ``parallelize_model``: the ``impl`` switch, and a CPU-offload request
(``fsdp2.offload_policy``), which only torch FSDP2 serves, so the recipes build real (not meta)
weights for it."""

from __future__ import annotations

import pytest

from mvp_engine.config.schema import BaseBackendKwargsConfig
from mvp_engine.distributed.parallelize import resolve_impl


def test_default_is_native_and_torch_is_kept():
    assert resolve_impl({}) == "native"
    assert resolve_impl({"impl": "torch"}) == "torch"
    assert resolve_impl(BaseBackendKwargsConfig()) == "native"


def test_offload_request_goes_to_torch_fsdp2():
    assert resolve_impl({"fsdp2": {"offload_policy": True}}) == "torch"
    assert resolve_impl({"impl": "torch", "fsdp2": {"offload_policy": True}}) == "torch"
    assert resolve_impl({"fsdp2": {"offload_policy": False}}) == "native"
    cfg = BaseBackendKwargsConfig()
    cfg.fsdp2.offload_policy = True
    assert resolve_impl(cfg) == "torch"


def test_unknown_impl_is_refused():
    with pytest.raises(ValueError, match="native' or 'torch"):
        resolve_impl({"impl": "jax"})


def test_recipe_builds_real_weights_when_offload_is_requested(tmp_path):
    from pathlib import Path

    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = Path(__file__).resolve().parent.parent / "recipes" / "qwen3"
    import_recipe_modules(root)
    over = ("model.pretrained_model_name_or_path=mvp/qwen3-tiny", "log.backends=[terminal]")
    plain = load_smoke_test_config(root, "synthetic_8b", output_dir=tmp_path, run_id="a", config_overrides=over)
    offload = load_smoke_test_config(root, "synthetic_8b", output_dir=tmp_path, run_id="b",
                                     config_overrides=over + ("parallel.backend_kwargs.fsdp2.offload_policy=true",))
    engine_cls = ENGINE_REGISTRY.get(plain["engine"])
    for cfg, native in ((plain, True), (offload, False)):
        eng = engine_cls.__new__(engine_cls)
        eng.config = eng.prepare_config(cfg)
        assert eng._native() is native
