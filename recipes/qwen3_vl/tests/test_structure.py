"""Structure tests of the qwen3_vl recipe."""

from pathlib import Path

from mvp_engine.testing.recipe_checks import BASE_FILES, check_config_structure, check_file_structure

RECIPE_ROOT = Path(__file__).resolve().parent.parent
SCHEMA_MODULE = "recipes.qwen3_vl.configs.schema"
CONFIG_CLASS = "Qwen3VLConfig"
EXPECTED_FILES = BASE_FILES + ('configs/train.yaml', 'model/qwen3_vl.py', 'model/packing/prepare.py', 'model/packing/qwen3_vl.py', 'dataset/__init__.py', 'utils/misc.py')


def test_file_structure():
    check_file_structure(RECIPE_ROOT, EXPECTED_FILES)


def test_config_structure():
    check_config_structure(RECIPE_ROOT, SCHEMA_MODULE, CONFIG_CLASS)
