"""Command-line entry point (reference: mvp_engine/launch.py:1-164).

    torchrun --nproc-per-node N -m mvp_engine.launch --config recipes/<r>/configs/<c>.yaml [k=v ...]

The recipe owning the config file is located under ``recipes/`` and every
module in it is imported (skipping ``_*``, ``tests`` and ``conftest`` and any
git-ignored file) so its engines register themselves.  The config is the
engine default YAML, merged under the recipe YAML, merged under the dotlist
overrides; ``workflow`` (default ``train``) selects ``engine.train()``,
``engine.evaluate()`` or any other engine method.  The process group is torn
down in ``finally``.
"""

from __future__ import annotations

import argparse
import importlib
import subprocess
import sys
from pathlib import Path
from collections.abc import Mapping
from typing import Optional, Sequence, Union

PROJECT_ROOT = Path(__file__).resolve().parent.parent
RECIPES_ROOT = PROJECT_ROOT / "recipes"
_PATCHED = False


def _apply_runtime_patches() -> None:
    global _PATCHED
    if not _PATCHED:
        from .patches import apply_all_patches

        apply_all_patches()
        _PATCHED = True


def find_recipe_dir(config_path: Path) -> Optional[Path]:
    try:
        rel = config_path.resolve().relative_to(RECIPES_ROOT)
    except ValueError:
        return None
    if len(rel.parts) < 2:
        return None
    d = RECIPES_ROOT / rel.parts[0]
    return d if d.is_dir() else None


def _not_ignored(paths: list[Path]) -> list[Path]:
    if not paths:
        return []
    try:
        rels = [p.resolve().relative_to(PROJECT_ROOT).as_posix() for p in paths]
    except ValueError:
        return paths
    try:
        r = subprocess.run(["git", "check-ignore", "--no-index", "--stdin"], input="\n".join(rels),
                           capture_output=True, cwd=PROJECT_ROOT, text=True, check=False)
    except (FileNotFoundError, OSError):
        return paths
    if r.returncode not in (0, 1):
        return paths
    ignored = {ln.strip() for ln in r.stdout.splitlines() if ln.strip()}
    return [p for p, rel in zip(paths, rels) if rel not in ignored]


def import_recipe_modules(recipe_dir: Path) -> None:
    packaged = (RECIPES_ROOT / "__init__.py").exists() and (recipe_dir / "__init__.py").exists()
    root = PROJECT_ROOT if packaged else recipe_dir.parent
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    files = sorted(p for p in recipe_dir.glob("**/*.py")
                   if not p.name.startswith("_") and p.name != "conftest.py" and "tests" not in p.parts)
    for f in _not_ignored(files):
        importlib.import_module(".".join(f.relative_to(root).with_suffix("").parts))


def _plain_dict(config) -> dict:
    """An OmegaConf / mapping-like config as nested plain dicts."""
    try:
        from omegaconf import OmegaConf

        return OmegaConf.to_container(config, resolve=True)
    except ImportError:
        return {k: _plain_dict(v) if hasattr(v, "keys") else v for k, v in config.items()}


def run(config: dict) -> object:
    """Build the configured engine and dispatch its workflow; returns the engine."""
    from .engine import ENGINE_REGISTRY

    _apply_runtime_patches()
    engine = ENGINE_REGISTRY.get(config.get("engine", "Engine"))(config)
    workflow = config.get("workflow", "train")
    if workflow == "train":
        engine.train()
    elif workflow == "evaluate":
        engine.evaluate()
    elif hasattr(engine, workflow):
        getattr(engine, workflow)()
    else:
        raise ValueError(f"Unknown workflow: {workflow}")
    return engine


def main(config: Optional[Union[Mapping, Sequence[str]]] = None) -> None:
    """Launcher entry.  ``config`` is either an already composed config (a mapping, as the reference's
    Hydra-decorated ``main(config)`` receives it; it is merged over ``config/default.yaml``) or the
    command-line arguments (``--config <yaml>`` plus dotlist overrides; ``None`` = ``sys.argv``)."""
    from .config.loader import compose_config, deep_merge, load_yaml

    if isinstance(config, Mapping) or hasattr(config, "keys"):
        composed = config if isinstance(config, dict) else _plain_dict(config)
        run(deep_merge(load_yaml(Path(__file__).parent / "config" / "default.yaml"), composed))
        return
    argv = config
    parser = argparse.ArgumentParser(description="mvp_engine launcher")
    parser.add_argument("--config", required=True, help="Path to YAML config file")
    args, overrides = parser.parse_known_args(argv)
    cfg_path = Path(args.config).resolve()
    recipe = find_recipe_dir(cfg_path)
    if recipe is not None:
        import_recipe_modules(recipe)
    # Hydra-style flags are accepted and ignored (the reference appends them itself).
    overrides = [o for o in overrides if not o.startswith(("hydra.", "hydra/", "--config-"))]
    config = compose_config(cfg_path, overrides)
    try:
        run(config)
    except Exception as exc:
        from .utils.log import simple_info

        simple_info(f"Exception occurred: {exc}", "error")
        raise
    finally:
        try:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:
            pass


if __name__ == "__main__":
    main()
