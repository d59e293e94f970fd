"""Windowed metric buffers with optional cross-rank reduction over a gloo group
(reference: mvp_engine/utils/log/metric.py:18-237)."""

from __future__ import annotations

import math
from typing import Dict, List, Literal, Optional, TypedDict, Union

import torch
import torch.distributed as dist

Value = Optional[Union[int, float, str, torch.Tensor]]


class Metric:
    """Keeps the last ``accumulation_size`` values; reduces them to a mean or sum.

    String values switch the metric to "last value" mode.  With ``support_nan``
    off, a NaN update repeats the previous value.  When ``distributed`` and a
    process group is set, sums and counts are all-reduced so every rank logs
    the global figure.
    """

    def __init__(self, accumulation_size: int = 20, distributed: bool = False, support_nan: bool = True,
                 dist_group: Optional[dist.ProcessGroup] = None) -> None:
        self._buf: List[Optional[Union[float, str]]] = []
        self._size = int(accumulation_size)
        self._distributed = distributed
        self._support_nan = support_nan
        self._group = dist_group
        self._is_string = False

    def update(self, value: Value) -> None:
        if value is None:
            self._buf.append(None)
        elif isinstance(value, str):
            self._is_string = True
            self._buf.append(value)
        else:
            if not isinstance(value, (int, float, torch.Tensor)):
                raise TypeError(f"Metric only supports int, float, str, torch.Tensor or None, got {type(value)}")
            v = float(value.detach().float().item()) if torch.is_tensor(value) else float(value)
            if math.isnan(v) and not self._support_nan:
                prev = self._buf[-1] if self._buf else None
                self._buf.append(prev)
            else:
                self._buf.append(v)
        overflow = len(self._buf) - (self._size + 1)
        if overflow > 0:
            del self._buf[:overflow]

    def clear(self) -> None:
        self._buf = []

    def _window(self) -> list:
        return [v for v in self._buf[-self._size:] if v is not None]

    def _reduce(self, total: float, count: float) -> tuple[float, float]:
        if self._distributed and self._group is not None:
            t = torch.tensor([total, count], dtype=torch.float64)
            dist.all_reduce(t, group=self._group)
            return float(t[0]), float(t[1])
        return total, count

    def mean(self) -> Union[float, str]:
        vals = self._window()
        if not vals:
            return "" if self._is_string else 0.0
        if self._is_string:
            return vals[-1]
        total, count = self._reduce(float(sum(vals)), float(len(vals)))
        return total / count if count else 0.0

    def sum(self) -> Union[float, str]:
        vals = self._window()
        if not vals:
            return "" if self._is_string else 0.0
        if self._is_string:
            return vals[-1]
        total, _ = self._reduce(float(sum(vals)), float(len(vals)))
        return total


class MetricEntry(TypedDict):
    """One named metric of a :class:`MetricAggregator`: its buffer, emission interval and update count."""

    metric: Metric
    interval: int
    update_count: int


class MetricAggregator:
    """Named metrics with an emission interval: a metric is reported every ``interval`` updates."""

    def __init__(self, dist_group: Optional[dist.ProcessGroup] = None, default_interval: int = 20,
                 default_accumulation_size: int = 20) -> None:
        self._metrics: Dict[str, MetricEntry] = {}
        self._group = dist_group
        self._interval = int(default_interval)
        self._acc = int(default_accumulation_size)

    def add(self, name: str, accumulation_size: Optional[int] = None, interval: Optional[int] = None,
            distributed: Optional[bool] = None, support_nan: bool = True) -> None:
        if name in self._metrics:
            return
        self._metrics[name] = MetricEntry(
            metric=Metric(accumulation_size or self._acc,
                          bool(distributed) if distributed is not None else self._group is not None,
                          support_nan, self._group),
            interval=int(interval or self._interval),
            update_count=0,
        )

    def __contains__(self, name: str) -> bool:
        return name in self._metrics

    def update(self, metrics: Dict[str, Value]) -> None:
        for name, value in metrics.items():
            if name not in self._metrics:
                self.add(name)
            entry = self._metrics[name]
            entry["metric"].update(value)
            entry["update_count"] += 1

    def collect(self, metric_names: Optional[List[str]] = None,
                accumulate: Literal["mean", "sum"] = "mean") -> Dict[str, Union[float, str]]:
        """Aggregated values of the metrics whose interval has elapsed.

        Every rank takes the same collection decisions (counts advance in
        lock-step), so distributed reductions stay matched across ranks.
        """
        names = metric_names if metric_names is not None else list(self._metrics)
        out: Dict[str, Union[float, str]] = {}
        for name in names:
            entry = self._metrics.get(name)
            if entry is None or entry["update_count"] % entry["interval"] != 0:
                continue
            m = entry["metric"]
            out[name] = m.mean() if accumulate == "mean" else m.sum()
        return out

    def collect_all(self, accumulate: Literal["mean", "sum"] = "mean") -> Dict[str, Union[float, str]]:
        return {n: (e["metric"].mean() if accumulate == "mean" else e["metric"].sum())
                for n, e in self._metrics.items()}
