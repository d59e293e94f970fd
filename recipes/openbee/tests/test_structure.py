"""Structure tests of the openbee recipe."""

from pathlib import Path

from mvp_engine.testing.recipe_checks import BASE_FILES, check_config_structure, check_file_structure

RECIPE_ROOT = Path(__file__).resolve().parent.parent
SCHEMA_MODULE = "recipes.openbee.configs.schema"
CONFIG_CLASS = "OpenBeeConfig"
EXPECTED_FILES = BASE_FILES + ('configs/stage1.yaml', 'configs/stage2.yaml', 'configs/stage3.yaml')


def test_file_structure():
    check_file_structure(RECIPE_ROOT, EXPECTED_FILES)


def test_config_structure():
    check_config_structure(RECIPE_ROOT, SCHEMA_MODULE, CONFIG_CLASS)
