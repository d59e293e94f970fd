"""Logger: windowed metrics (reduced over a gloo side group) fanned out to the log backends.

Public API of the reference's ``Logger`` (``mvp_engine/utils/log/logger.py:23-200``): the
constructor arguments, ``log_config`` / ``log_metrics`` / ``add_metric(s)`` / ``summary`` /
``destroy`` and the four message levels.  Metric reduction across ranks runs on a separate
gloo group so that logging never enqueues work on the NCCL communicator the training step
uses.  Every call is a fan-out: the same method is called on each backend in order.
"""

from __future__ import annotations

import os
from enum import IntEnum
from typing import Any, List, Mapping, Optional, Union

import torch
import torch.distributed as dist

from ...distributed.utils import get_world_size
from .backend.backend import Backend
from .metric import MetricAggregator


class LogLevel(IntEnum):
    DEBUG = 10
    INFO = 20
    WARNING = 30
    ERROR = 40


_LEVEL_NAMES = {"debug": LogLevel.DEBUG, "info": LogLevel.INFO, "warn": LogLevel.WARNING,
                "warning": LogLevel.WARNING, "error": LogLevel.ERROR}


def parse_log_level(level: str) -> LogLevel:
    found = _LEVEL_NAMES.get(str(level).strip().lower())
    if found is None:
        raise ValueError(f"Invalid log level '{level}'. Supported levels: {', '.join(_LEVEL_NAMES)}.")
    return found


def _metric_side_group() -> Optional[dist.ProcessGroup]:
    if get_world_size() <= 1 or not dist.is_initialized():
        return None
    os.environ.setdefault("GLOO_LOG_LEVEL", "ERROR")
    return dist.new_group(backend="gloo")


class Logger:
    def __init__(self, backends: List[Backend], interval: int = 20, accumulation_size: int = 20,
                 level: LogLevel = LogLevel.INFO) -> None:
        self.backends = list(backends)
        self.level = level
        self.step = 0
        self.total_steps: Optional[int] = None
        self.metrics = MetricAggregator(dist_group=_metric_side_group(), default_interval=interval,
                                        default_accumulation_size=accumulation_size)

    def _fan_out(self, method: str, *args: Any, **kwargs: Any) -> None:
        for backend in self.backends:
            getattr(backend, method)(*args, **kwargs)

    # ------------------------------------------------------------- metrics
    def log_config(self, config: dict) -> None:
        self._fan_out("log_config", config)

    def add_metric(self, name: str, accumulation_size: Optional[int] = None, interval: Optional[int] = None,
                   distributed: Optional[bool] = None, support_nan: bool = True) -> None:
        self.metrics.add(name, accumulation_size, interval, distributed, support_nan)

    def add_metrics(self, names: List[str], accumulation_size: Optional[int] = None, interval: Optional[int] = None,
                    distributed: Optional[bool] = None, support_nan: bool = True) -> None:
        for name in names:
            self.metrics.add(name, accumulation_size, interval, distributed, support_nan)

    def log_metrics(self, metrics: Mapping[str, Union[int, float, str, torch.Tensor]], step: int,
                    epoch: Optional[int] = None, total_steps: Optional[int] = None) -> None:
        """Feed this step's values into the windows; backends receive whatever is due at this step."""
        self.step = step
        if total_steps is not None:
            self.total_steps = total_steps
        self.metrics.update(dict(metrics))
        due = self.metrics.collect(metric_names=list(metrics))
        if due:
            self._fan_out("log_metrics", due, step, epoch, self.total_steps)

    def summary(self) -> None:
        self._fan_out("log_metrics", self.metrics.collect_all(), self.step, total_steps=self.total_steps)

    def destroy(self) -> None:
        self._fan_out("destroy")
        from . import logger as proxy

        if proxy._instance is self:
            proxy._instance = None

    # ------------------------------------------------------------ messages
    def _message(self, level: LogLevel, message: str) -> None:
        if level >= self.level:
            self._fan_out(level.name.lower(), message)

    def debug(self, message: str) -> None:
        self._message(LogLevel.DEBUG, message)

    def info(self, message: str) -> None:
        self._message(LogLevel.INFO, message)

    def warning(self, message: str) -> None:
        self._message(LogLevel.WARNING, message)

    def error(self, message: str) -> None:
        self._message(LogLevel.ERROR, message)
