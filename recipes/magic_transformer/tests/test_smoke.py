"""Smoke test of the magic_transformer recipe (runs with --run-smoke; default config 'train')."""

from pathlib import Path

import pytest

from mvp_engine.testing.recipe_checks import run_recipe_smoke

RECIPE_ROOT = Path(__file__).resolve().parent.parent


def test_smoke(run_smoke, world_size, config_name, config_overrides, tmp_path):
    if not run_smoke:
        pytest.skip("pass --run-smoke (needs the recipe's hardware)")
    run_recipe_smoke(RECIPE_ROOT, config_name or "train", world_size=world_size, output_dir=tmp_path,
                     overrides=("loop.total_steps=2",) + tuple(config_overrides))
