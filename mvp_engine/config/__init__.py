"""Configuration schema and YAML/CLI composition."""

from .loader import apply_dotlist, compose_config, deep_merge, load_yaml, to_container
from .schema import BaseEngineConfig

__all__ = ["BaseEngineConfig", "compose_config", "apply_dotlist", "deep_merge", "load_yaml", "to_container"]
