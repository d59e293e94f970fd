"""YAML + command-line config composition.

The launch contract is the reference's (``--config path.yaml k=v ...``, the
engine default YAML merged underneath the recipe YAML, then the dotlist;
reference: mvp_engine/launch.py:98-164).  When OmegaConf is importable it is
used for the merge; otherwise a built-in deep merge with the same rules runs:

* mappings merge key by key, every other value (lists included) replaces;
* ``a.b.c=value`` sets a nested key, the value parsed as YAML
  (``true``, ``1e-3``, ``[1,2]``, ``null``);
* ``+a.b=value`` adds a key, ``++a.b=value`` adds or overrides, ``~a.b`` deletes.
* ``${a.b}`` interpolations in string values resolve against the merged tree.
"""

from __future__ import annotations

import copy
import re
from pathlib import Path
from typing import Any, Iterable, Mapping

import yaml

DEFAULT_CONFIG_PATH = Path(__file__).with_name("default.yaml")
_INTERP = re.compile(r"\$\{([^}]+)\}")


def load_yaml(path: str | Path) -> dict:
    with open(path) as f:
        data = yaml.safe_load(f) or {}
    if not isinstance(data, dict):
        raise ValueError(f"{path}: top level must be a mapping")
    return data


def deep_merge(base: Mapping, override: Mapping) -> dict:
    out = copy.deepcopy(dict(base))
    for k, v in override.items():
        if isinstance(v, Mapping) and isinstance(out.get(k), Mapping):
            out[k] = deep_merge(out[k], v)
        else:
            out[k] = copy.deepcopy(v)
    return out


def _set(tree: dict, dotted: str, value: Any, *, must_exist: bool | None) -> None:
    keys = dotted.split(".")
    node = tree
    for k in keys[:-1]:
        if k not in node or not isinstance(node[k], dict):
            if must_exist:
                raise KeyError(f"override {dotted!r}: key {k!r} does not exist (use +{dotted}=...)")
            node[k] = {}
        node = node[k]
    last = keys[-1]
    if must_exist is True and last not in node:
        raise KeyError(f"override {dotted!r}: key does not exist (use +{dotted}=...)")
    if must_exist is False and last in node:
        raise KeyError(f"override +{dotted}: key already exists (use {dotted}=... or ++{dotted}=...)")
    node[last] = value


def _delete(tree: dict, dotted: str) -> None:
    keys = dotted.split(".")
    node = tree
    for k in keys[:-1]:
        node = node[k]
    node.pop(keys[-1], None)


def _parse_value(raw: str) -> Any:
    """YAML scalar/collection parsing; YAML 1.1 leaves '1e-3' a string, so numbers are retried."""
    if raw == "":
        return ""
    value = yaml.safe_load(raw)
    if isinstance(value, str):
        for cast in (int, float):
            try:
                return cast(value)
            except ValueError:
                continue
    return value


def apply_dotlist(tree: dict, overrides: Iterable[str]) -> dict:
    out = copy.deepcopy(tree)
    for item in overrides:
        item = item.strip()
        if not item:
            continue
        if item.startswith("~"):
            _delete(out, item[1:].split("=", 1)[0])
            continue
        if "=" not in item:
            raise ValueError(f"override {item!r} must look like key=value")
        key, raw = item.split("=", 1)
        value = _parse_value(raw)
        if key.startswith("++"):
            _set(out, key[2:], value, must_exist=None)
        elif key.startswith("+"):
            _set(out, key[1:], value, must_exist=False)
        else:
            _set(out, key, value, must_exist=None)
    return out


def _lookup(tree: Mapping, dotted: str) -> Any:
    node: Any = tree
    for k in dotted.split("."):
        node = node[k]
    return node


def resolve_interpolations(tree: Any, root: Mapping | None = None, depth: int = 0) -> Any:
    root = tree if root is None else root
    if depth > 16:
        raise ValueError("config interpolation is too deep (cycle?)")
    if isinstance(tree, dict):
        return {k: resolve_interpolations(v, root, depth) for k, v in tree.items()}
    if isinstance(tree, list):
        return [resolve_interpolations(v, root, depth) for v in tree]
    if isinstance(tree, str):
        full = _INTERP.fullmatch(tree)
        if full:
            return resolve_interpolations(_lookup(root, full.group(1).strip()), root, depth + 1)
        return _INTERP.sub(lambda m: str(resolve_interpolations(_lookup(root, m.group(1).strip()), root, depth + 1)),
                           tree)
    return tree


def compose_config(config_path: str | Path | None, overrides: Iterable[str] = (), *,
                   defaults: str | Path | None = DEFAULT_CONFIG_PATH) -> dict:
    """default.yaml <- recipe YAML <- dotlist, then interpolation; returns a plain dict."""
    tree = load_yaml(defaults) if defaults else {}
    if config_path is not None:
        tree = deep_merge(tree, load_yaml(config_path))
    tree = apply_dotlist(tree, list(overrides))
    return resolve_interpolations(tree)


def to_container(cfg: Any) -> Any:
    """Plain-python view of a dict / OmegaConf object / pydantic model."""
    if hasattr(cfg, "model_dump"):
        return cfg.model_dump()
    try:  # OmegaConf DictConfig, when installed
        from omegaconf import OmegaConf  # type: ignore

        if OmegaConf.is_config(cfg):
            return OmegaConf.to_container(cfg, resolve=True)
    except ImportError:
        pass
    return copy.deepcopy(cfg)
