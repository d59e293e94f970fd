"""Global logger.

``from mvp_engine.utils.log import logger`` works before :func:`init_logger`:
the proxy forwards to the active :class:`Logger` once one exists and falls back
to :func:`simple_info` printing until then
(reference: mvp_engine/utils/log/__init__.py:17-165).
"""

from __future__ import annotations

import os
import sys
from datetime import datetime
from typing import List, Optional

from .logger import Logger, LogLevel, parse_log_level


def _env_level() -> LogLevel:
    raw = os.environ.get("LOG_LEVEL")
    if not raw:
        return LogLevel.INFO
    try:
        return parse_log_level(raw)
    except ValueError:
        print(f"[mvp_engine] invalid LOG_LEVEL={raw!r}; using INFO", file=sys.stderr)
        return LogLevel.INFO


def simple_info(message: str, level: str = "info") -> None:
    """Rank-0 print with a timestamp; usable before any logger exists."""
    from ...distributed.utils import get_rank

    if get_rank() != 0:
        return
    lv = parse_log_level(level) if level else LogLevel.INFO
    if lv < _env_level():
        return
    print(f"[{datetime.now():%H:%M:%S}] {lv.name:<7} {message}", flush=True)


class LoggerProxy:
    """Stand-in object bound at import time; resolves to the live Logger."""

    def __getattr__(self, name):
        inst = type(self).__dict__.get("_inst")
        if inst is not None:
            return getattr(inst, name)
        if name in ("info", "debug", "warning", "error"):
            return lambda msg: simple_info(str(msg), name)
        if name in ("log_metrics", "log_config", "add_metric", "add_metrics", "summary", "destroy"):
            return lambda *a, **k: None
        raise AttributeError(name)

    def __bool__(self) -> bool:
        return type(self)._instance is not None

    @property
    def _instance(self):  # type: ignore[override]
        return type(self).__dict__.get("_inst")

    @_instance.setter
    def _instance(self, value):
        type(self)._inst = value


logger = LoggerProxy()


def get_logger() -> Optional[Logger]:
    return LoggerProxy.__dict__.get("_inst")


def init_logger(backends: List, interval: int = 20, accumulation_size: Optional[int] = None,
                level: Optional[LogLevel] = None) -> LoggerProxy:
    inst = Logger(backends, interval=interval,
                  accumulation_size=accumulation_size if accumulation_size is not None else interval,
                  level=level if level is not None else _env_level())
    logger._instance = inst
    return logger


def __getattr__(name: str):
    # the backend base class for custom backends, imported on first use (the backends import this module)
    if name == "Backend":
        from .backend.backend import Backend

        return Backend
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = ["Backend", "Logger", "LogLevel", "logger", "init_logger", "get_logger", "simple_info", "parse_log_level"]
