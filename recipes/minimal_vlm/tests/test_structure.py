"""Structure tests of the minimal_vlm recipe."""

from pathlib import Path

from mvp_engine.testing.recipe_checks import BASE_FILES, check_config_structure, check_file_structure

RECIPE_ROOT = Path(__file__).resolve().parent.parent
SCHEMA_MODULE = "recipes.minimal_vlm.configs.schema"
CONFIG_CLASS = "MinimalVLMConfig"
EXPECTED_FILES = BASE_FILES + ('configs/train.yaml', 'dataset/preprocess.py', 'dataset/collator.py')


def test_file_structure():
    check_file_structure(RECIPE_ROOT, EXPECTED_FILES)


def test_config_structure():
    check_config_structure(RECIPE_ROOT, SCHEMA_MODULE, CONFIG_CLASS)
