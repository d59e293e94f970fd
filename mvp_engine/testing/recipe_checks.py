"""Shared recipe test harness (reference: tests/templates/*.template and recipes/*/tests/*).

``check_file_structure`` / ``check_config_structure`` back every recipe's
``tests/test_structure.py``; ``run_recipe_smoke`` backs ``tests/test_smoke.py``
(spawned ranks, one engine step loop with the recipe's skill asserts
injected).  Skill assert modules live in ``recipes/<r>/tests/skills/<id>/asserts.py``
and may define ``test_file_structure(recipe_root)``, ``test_config_structure(config)``,
``test_engine_structure(engine_class)`` and ``assert_<phase>_{start,end}`` hooks.
"""

from __future__ import annotations

import importlib
from pathlib import Path
from typing import Any, Iterable, Optional

import yaml

from .utils import (inject_engine_assert_hooks, load_recipe_skill_asserts, load_smoke_test_config,
                    spawn_workers)

BASE_FILES = ("README.md", "__init__.py", "configs/__init__.py", "configs/schema.py", "engine/__init__.py",
              "model/__init__.py")


def check_file_structure(recipe_root: Path, expected: Iterable[str] = BASE_FILES) -> None:
    recipe_root = Path(recipe_root)
    for rel in expected:
        assert (recipe_root / rel).exists(), f"{rel} does not exist in {recipe_root.name}"
    for mod in load_recipe_skill_asserts(recipe_root):
        if hasattr(mod, "test_file_structure"):
            mod.test_file_structure(recipe_root)


def check_config_structure(recipe_root: Path, schema_module: str, class_name: str) -> list[Any]:
    """Every ``configs/*.yaml`` merged over the defaults validates against the recipe schema and names a
    registered engine whose ``ConfigClass`` is that schema."""
    from ..config.loader import deep_merge, load_yaml
    from ..engine import ENGINE_REGISTRY
    from ..launch import import_recipe_modules

    recipe_root = Path(recipe_root)
    import_recipe_modules(recipe_root)
    cls = getattr(importlib.import_module(schema_module), class_name)
    default = load_yaml(Path(__file__).resolve().parent.parent / "config" / "default.yaml")
    skill_mods = load_recipe_skill_asserts(recipe_root)
    out = []
    paths = sorted((recipe_root / "configs").glob("*.yaml"))
    assert paths, f"{recipe_root.name} has no configs"
    for p in paths:
        raw = deep_merge(default, yaml.safe_load(p.read_text()))
        cfg = cls.model_validate(raw)
        engine_cls = ENGINE_REGISTRY.get(cfg.engine)
        assert issubclass(cls, engine_cls.ConfigClass) or engine_cls.ConfigClass is cls, p.name
        for mod in skill_mods:
            if hasattr(mod, "test_config_structure"):
                mod.test_config_structure(cfg.model_dump())
            if hasattr(mod, "test_engine_structure"):
                mod.test_engine_structure(engine_cls)
        out.append(cfg)
    return out


def _smoke_worker(rank, world, port, recipe_root, config_name, output_dir, overrides):
    from ..engine import ENGINE_REGISTRY
    from ..launch import import_recipe_modules

    import_recipe_modules(Path(recipe_root))
    cfg = load_smoke_test_config(Path(recipe_root), config_name, output_dir=Path(output_dir),
                                 config_overrides=tuple(overrides))
    engine = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    inject_engine_assert_hooks(engine, load_recipe_skill_asserts(Path(recipe_root)))
    engine.train()
    return getattr(engine, "last_logs", None)


def run_recipe_smoke(recipe_root: Path, config_name: str, *, world_size: int, output_dir: Path,
                     overrides: Optional[Iterable[str]] = None, timeout: float = 3600.0) -> list[Any]:
    return spawn_workers(_smoke_worker, world_size, str(recipe_root), config_name, str(output_dir),
                         list(overrides or ()), timeout=timeout)
