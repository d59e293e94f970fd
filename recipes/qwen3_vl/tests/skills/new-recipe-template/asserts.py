"""Skill asserts: the layout every recipe shares.

Copy to ``recipes/<recipe>/tests/skills/new-recipe-template/asserts.py``.  A recipe is a package with a
pydantic config schema, YAML configs that validate against it, an engine registered under the name the
configs give, and the model / data glue it needs; tests live beside it.
"""

from mvp_engine.testing.skill_checks import phase_source

_FILES = ("README.md", "__init__.py", "configs/__init__.py", "configs/schema.py", "engine/__init__.py",
          "model/__init__.py", "tests/test_structure.py", "tests/test_smoke.py")
_PHASES = ("prepare_model", "prepare_optimizer", "prepare_scheduler", "prepare_dataloader", "forward_step",
           "backward_step", "optimizer_step", "train_post_step")


def test_file_structure(recipe_root):
    for rel in _FILES:
        assert (recipe_root / rel).exists(), f"recipe {recipe_root.name} lacks {rel}"
    assert list((recipe_root / "configs").glob("*.yaml")), f"recipe {recipe_root.name} has no configs/*.yaml"


def test_engine_structure(engine_class):
    from mvp_engine.engine import ENGINE_REGISTRY, Engine

    assert issubclass(engine_class, Engine), "a recipe engine derives from mvp_engine.engine.Engine"
    assert ENGINE_REGISTRY.get(engine_class.__name__) is engine_class, "register the engine (ENGINE_REGISTRY)"
    assert getattr(engine_class, "ConfigClass", None) is not None, "the engine names its config schema"
    for phase in _PHASES:
        owner = next(k for k in engine_class.__mro__ if phase in k.__dict__)
        assert owner is not Engine or phase in ("forward_step", "backward_step", "optimizer_step", "train_post_step"), (
            f"{phase} has no default: the recipe engine must implement it")
        assert phase_source(engine_class, phase), phase
