"""Logger: metric aggregation over a gloo side group + fan-out to backends
(reference: mvp_engine/utils/log/logger.py:23-200)."""

from __future__ import annotations

import os
from enum import IntEnum
from typing import List, Mapping, Optional, Union

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


def parse_log_level(level: str) -> LogLevel:
    key = str(level).strip().upper()
    if key == "WARN":
        key = "WARNING"
    if key not in LogLevel.__members__:
        raise ValueError(f"Invalid log level: {level}")
    return LogLevel[key]


class Logger:
    def __init__(self, backends: List[Backend], interval: int = 20, accumulation_size: int = 20,
                 level: LogLevel = LogLevel.INFO) -> None:
        group = None
        if get_world_size() > 1 and dist.is_initialized():
            os.environ.setdefault("GLOO_LOG_LEVEL", "ERROR")
            group = dist.new_group(backend="gloo")
        self.metrics = MetricAggregator(dist_group=group, default_interval=interval,
                                        default_accumulation_size=accumulation_size)
        self.step = 0
        self.total_steps: Optional[int] = None
        self.backends = list(backends)
        self.level = level

    def log_config(self, config: dict) -> None:
        for b in self.backends:
            b.log_config(config)

    def summary(self) -> None:
        collected = self.metrics.collect_all()
        for b in self.backends:
            b.log_metrics(collected, self.step, total_steps=self.total_steps)

    def add_metric(self, name: str, accumulation_size: Optional[int] = None, interval: Optional[int] = None,
                   distributed: Optional[bool] = None, support_nan: bool = True) -> None:
        self.metrics.add(name, accumulation_size, interval, distributed, support_nan)

    def add_metrics(self, names: List[str], accumulation_size: Optional[int] = None, interval: Optional[int] = None,
                    distributed: Optional[bool] = None, support_nan: bool = True) -> None:
        for n in names:
            self.add_metric(n, accumulation_size, interval, distributed, support_nan)

    def log_metrics(self, metrics: Mapping[str, Union[int, float, str, torch.Tensor]], step: int,
                    epoch: Optional[int] = None, total_steps: Optional[int] = None) -> None:
        self.metrics.update(dict(metrics))
        self.step = step
        if total_steps is not None:
            self.total_steps = total_steps
        collected = self.metrics.collect(metric_names=list(metrics.keys()))
        if collected:
            for b in self.backends:
                b.log_metrics(collected, step, epoch, self.total_steps)

    def destroy(self) -> None:
        for b in self.backends:
            b.destroy()
        from . import logger as proxy

        if proxy._instance is self:
            proxy._instance = None

    def _emit(self, level: LogLevel, method: str, message: str) -> None:
        if level < self.level:
            return
        for b in self.backends:
            getattr(b, method)(message)

    def debug(self, message: str) -> None:
        self._emit(LogLevel.DEBUG, "debug", message)

    def info(self, message: str) -> None:
        self._emit(LogLevel.INFO, "info", message)

    def warning(self, message: str) -> None:
        self._emit(LogLevel.WARNING, "warning", message)

    def error(self, message: str) -> None:
        self._emit(LogLevel.ERROR, "error", message)
