"""Config composition, schema validation, registry and mesh-shape inference (CPU)."""

import pytest

from mvp_engine.config.loader import apply_dotlist, compose_config, deep_merge, resolve_interpolations
from mvp_engine.config.schema import BaseEngineConfig
from mvp_engine.distributed.parallel_mesh import resolve_mesh_shape
from mvp_engine.utils.registry import Registry


def test_deep_merge_and_dotlist():
    base = {"a": {"b": 1, "c": [1, 2]}, "d": 1}
    merged = deep_merge(base, {"a": {"c": [3]}, "e": 2})
    assert merged == {"a": {"b": 1, "c": [3]}, "d": 1, "e": 2}
    out = apply_dotlist(merged, ["a.b=5", "+f.g=true", "~d", "a.c=[1,2,3]", "h=1e-3"])
    assert out["a"]["b"] == 5 and out["f"]["g"] is True and "d" not in out and out["a"]["c"] == [1, 2, 3]
    assert out["h"] == pytest.approx(1e-3)
    with pytest.raises(KeyError):
        apply_dotlist(out, ["+a.b=1"])


def test_interpolation():
    tree = resolve_interpolations({"x": 3, "y": "${x}", "z": "n=${x}"})
    assert tree == {"x": 3, "y": 3, "z": "n=3"}


def test_compose_recipe_config_validates(tmp_path):
    cfg = compose_config("recipes/qwen3/configs/train.yaml", ["optim.lr=1e-4", "parallel.mesh.context=2"])
    from recipes.qwen3.configs.schema import Qwen3Config

    c = Qwen3Config.model_validate(cfg)
    assert c.optim.lr == 1e-4 and c.parallel.mesh.context == 2 and c.engine == "Qwen3Engine"
    assert c.checkpoint.hf_enable is True


def test_schema_rejects_bad_mesh():
    with pytest.raises(Exception):
        BaseEngineConfig.model_validate({"parallel": {"mesh": {"shard": 0}}})


def test_batching_resolution():
    from recipes.qwen3.configs.schema import Qwen3Config

    c = Qwen3Config.model_validate({"optim": {"global_batch_size": 64, "gradient_accumulation_steps": -1},
                                    "data": {"batch_size": 1}})
    c.resolve_batching_config(data_parallel_world_size=8)
    assert c.optim.gradient_accumulation_steps == 8
    c = Qwen3Config.model_validate({"optim": {"global_batch_size": 64, "gradient_accumulation_steps": 2},
                                    "data": {"batch_size": -1}})
    c.resolve_batching_config(data_parallel_world_size=8)
    assert c.data.batch_size == 4
    c = Qwen3Config.model_validate({"optim": {"global_batch_size": 60, "gradient_accumulation_steps": -1},
                                    "data": {"batch_size": 1}})
    with pytest.raises(ValueError):
        c.resolve_batching_config(data_parallel_world_size=8)


def test_mesh_inference():
    assert resolve_mesh_shape({"replicate": 1, "shard": -1, "tensor": 2}, 8) == {"replicate": 1, "shard": 4,
                                                                                   "tensor": 2}
    with pytest.raises(ValueError):
        resolve_mesh_shape({"replicate": -1, "shard": -1}, 8)
    with pytest.raises(ValueError):
        resolve_mesh_shape({"replicate": 3, "shard": -1}, 8)
    with pytest.raises(ValueError):
        resolve_mesh_shape({"replicate": 2, "shard": 2}, 8)


def test_registry():
    r = Registry()

    @r.register()
    class A:
        pass

    @r.register("bee")
    def b():
        return 1

    @r.register
    class C:
        pass

    assert r.get("A") is A and r["bee"] is b and "C" in r
    with pytest.raises(KeyError):
        r.get("missing")


def _reference_yamls():
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent / "baseline" / "_ref" / "recipes"
    return sorted(root.glob("*/configs/*.yaml")) if root.is_dir() else []


@pytest.mark.skipif(not _reference_yamls(), reason="the reference is not installed under baseline/_ref")
@pytest.mark.parametrize("path", _reference_yamls(), ids=lambda p: f"{p.parts[-3]}/{p.name}")
def test_reference_recipe_yaml_validates_unchanged(path):
    """A recipe YAML of the reference, unmodified, composes with this engine's defaults and validates
    against the same-named recipe's schema here; its engine name is registered."""
    from pathlib import Path

    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules

    import_recipe_modules(Path(__file__).resolve().parent.parent / "recipes" / path.parts[-3])
    cfg = compose_config(str(path), [])
    engine_cls = ENGINE_REGISTRY.get(cfg["engine"])
    parsed = engine_cls.ConfigClass.model_validate(cfg)
    assert parsed.engine == cfg["engine"]
