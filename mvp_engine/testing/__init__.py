"""Test helpers: distributed env, worker spawning, smoke configs, engine hooks, fault injection."""

from .utils import (distributed_env, find_free_port, inject_engine_assert_hooks, inject_engine_hook,
                    load_recipe_skill_asserts, load_smoke_test_config, read_recipe_source, spawn_workers)

__all__ = ["distributed_env", "find_free_port", "inject_engine_assert_hooks", "inject_engine_hook",
           "load_recipe_skill_asserts", "load_smoke_test_config", "read_recipe_source", "spawn_workers"]
