"""Options of the recipe smoke tests (one definition for every recipe)."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_addoption(parser):
    parser.addoption("--run-smoke", action="store_true", default=False, help="run recipe smoke tests")
    parser.addoption("--world-size", type=int, default=1, help="ranks for smoke tests")
    parser.addoption("--config-name", default=None, help="recipe config (configs/<name>.yaml) for smoke tests")
    parser.addoption("--config-override", action="append", default=[], help="dotlist override (repeatable)")


@pytest.fixture
def run_smoke(request):
    return request.config.getoption("--run-smoke")


@pytest.fixture
def world_size(request):
    return request.config.getoption("--world-size")


@pytest.fixture
def config_name(request):
    return request.config.getoption("--config-name")


@pytest.fixture
def config_overrides(request):
    return tuple(request.config.getoption("--config-override"))
