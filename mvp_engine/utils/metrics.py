"""Windowed metric accumulation, locally and across ranks.

Public API of the reference's ``mvp_engine/utils/metrics.py:16-295`` (used by the
OpenBee recipe and by user engines): :class:`MetricAccumulator` (per-process
reducers, finalised to floats), :class:`DistributedMetric` and
:class:`DistributedMetricAccumulator` (local accumulation, then one collective
per reduction kind, cached as the global value).

Design: every reducer is a row of one table (how two values combine, whether the
update count divides the total at the end), so the local and the distributed
accumulators share the arithmetic.  Names accepted: ``sum``/``add``,
``mean``/``avg``, ``max``, ``last`` locally; ``sum``, ``max``, ``mean``/``avg``
and ``none`` across ranks.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Literal, Optional, Union

import torch
import torch.distributed as dist

ReducerName = Literal["sum", "last", "max", "mean"]
AccumulatorName = Literal["sum", "add", "last", "max", "mean", "avg"]
DistributedReducerName = Literal["sum", "max", "mean", "avg", "none"]

Value = Union[float, int, torch.Tensor]


def _maximum(a: Value, b: Value) -> Value:
    if isinstance(a, torch.Tensor) or isinstance(b, torch.Tensor):
        return torch.maximum(torch.as_tensor(a), torch.as_tensor(b))
    return max(a, b)


@dataclass(frozen=True)
class _Rule:
    combine: Callable[[Value, Value], Value]  # (running value, new value) -> running value
    divide_by_count: bool


_RULES: dict[str, _Rule] = {
    "sum": _Rule(lambda acc, v: acc + v, False),
    "mean": _Rule(lambda acc, v: acc + v, True),
    "max": _Rule(_maximum, False),
    "last": _Rule(lambda acc, v: v, False),
}
_LOCAL_ALIASES = {"add": "sum", "avg": "mean"}
_GLOBAL_ALIASES = {"avg": "mean"}
_GLOBAL_KINDS = ("sum", "max", "mean", "none")


def _local_rule_name(name: str) -> str:
    canon = _LOCAL_ALIASES.get(name, name)
    if canon not in _RULES:
        raise ValueError(f"Unsupported accumulation method: {name}")
    return canon


def _global_kind(name: str) -> str:
    canon = _GLOBAL_ALIASES.get(name, name)
    if canon not in _GLOBAL_KINDS:
        raise ValueError(f"Unsupported distributed reduce method: {name}")
    return canon


class _Running:
    """Running value + update count of one metric under one rule."""

    __slots__ = ("rule", "value", "count")

    def __init__(self, rule: str) -> None:
        self.rule = rule
        self.clear()

    def clear(self) -> None:
        self.value: Optional[Value] = None
        self.count = 0

    def add(self, v: Value) -> None:
        self.value = v if self.value is None else _RULES[self.rule].combine(self.value, v)
        self.count += 1

    def result(self) -> Optional[Value]:
        if self.value is None or self.count == 0:
            return None
        return self.value / self.count if _RULES[self.rule].divide_by_count else self.value


def _scalar_float(v: Value) -> float:
    if isinstance(v, torch.Tensor):
        if v.numel() != 1:
            raise ValueError("MetricAccumulator can only finalize scalar tensors to float.")
        return float(v.item())
    return float(v)


def _plain(v: Any) -> Value:
    if isinstance(v, torch.Tensor):
        return v.detach()
    if isinstance(v, (bool, int, float)):
        return float(v) if isinstance(v, bool) else v
    raise TypeError(f"Unsupported metric value type: {type(v).__name__}")


class MetricAccumulator:
    """Named metrics reduced over a window with ``sum`` / ``mean`` / ``max`` / ``last``."""

    def __init__(self, reducers: Optional[dict[str, ReducerName]] = None) -> None:
        self.reducers: dict[str, str] = {}
        self._running: dict[str, _Running] = {}
        for name, reducer in (reducers or {}).items():
            self.register(name, reducer)

    def register(self, name: str, reducer: ReducerName) -> None:
        if name in self.reducers:
            raise ValueError(f"Metric '{name}' is already registered.")
        if reducer not in _RULES:
            raise ValueError(f"Unsupported reducer '{reducer}' for metric '{name}'.")
        self.reducers[name] = reducer
        self._running[name] = _Running(reducer)

    def _slot(self, name: str) -> _Running:
        try:
            return self._running[name]
        except KeyError:
            raise KeyError(f"Metric '{name}' is not registered.") from None

    def reset(self) -> None:
        for slot in self._running.values():
            slot.clear()

    def update(self, **metrics: Any) -> None:
        for name, value in metrics.items():
            slot = self._slot(name)
            if value is not None:
                slot.add(_plain(value))

    def get(self, name: str) -> Optional[Value]:
        """The raw running value (the sum, for ``mean``)."""
        return self._slot(name).value

    def finalize(self) -> dict[str, float]:
        out = {}
        for name, slot in self._running.items():
            res = slot.result()
            if res is not None:
                out[name] = _scalar_float(res)
        return out


class DistributedMetric:
    """One scalar metric: accumulated on this rank, then reduced across ranks on demand."""

    def __init__(self, *, name: str, device: torch.device, accumulate: AccumulatorName,
                 reduce: DistributedReducerName) -> None:
        self.name = name
        self.device = torch.device(device)
        self.accumulate = _local_rule_name(accumulate)
        self.reduce = _global_kind(reduce)
        self._run = _Running(self.accumulate)
        self._global_value: Optional[float] = None

    def reset(self) -> None:
        self._run.clear()
        self._global_value = None

    def _tensor(self, v: Any) -> torch.Tensor:
        if isinstance(v, torch.Tensor):
            if v.numel() != 1:
                raise ValueError(f"Metric '{self.name}' only supports scalar tensors.")
            return v.detach().to(device=self.device, dtype=torch.float32).reshape(())
        if isinstance(v, (bool, int, float)):
            return torch.tensor(float(v), device=self.device, dtype=torch.float32)
        raise TypeError(f"Unsupported metric value type for '{self.name}': {type(v).__name__}")

    def update(self, value: Any) -> None:
        if value is None:
            return
        self._global_value = None
        if self.accumulate == "last":
            self._run.clear()  # "last" keeps one update: the newest
        self._run.add(self._tensor(value))

    def _local_tensor(self) -> torch.Tensor:
        if self._run.value is None:
            raise RuntimeError(f"Metric '{self.name}' has no local value.")
        return self._run.result()

    @property
    def local_value(self) -> float:
        return float(self._local_tensor().item())

    def set_global_tensor(self, value: torch.Tensor) -> None:
        self._global_value = float(value.item())

    @property
    def global_value(self) -> float:
        if self._global_value is None:
            raise RuntimeError(f"Metric '{self.name}' has not been reduced yet.")
        return self._global_value


class DistributedMetricAccumulator:
    """A set of :class:`DistributedMetric`, reduced together with one collective per reduction kind."""

    def __init__(self, device: torch.device) -> None:
        self.device = torch.device(device)
        self._metrics: dict[str, DistributedMetric] = {}

    def register(self, name: str, *, accumulate: AccumulatorName = "sum",
                 reduce: DistributedReducerName = "sum") -> None:
        if name in self._metrics:
            raise ValueError(f"Metric '{name}' is already registered.")
        self._metrics[name] = DistributedMetric(name=name, device=self.device, accumulate=accumulate, reduce=reduce)

    def update(self, **metrics: Any) -> None:
        for name, value in metrics.items():
            if name not in self._metrics:
                raise KeyError(f"Metric '{name}' is not registered.")
            self._metrics[name].update(value)

    def reduce_all(self) -> None:
        by_kind: dict[str, list[DistributedMetric]] = {}
        for m in self._metrics.values():
            by_kind.setdefault(m.reduce, []).append(m)
        live = dist.is_available() and dist.is_initialized()
        for kind in _GLOBAL_KINDS:  # fixed order: every rank issues the same collectives
            group = by_kind.get(kind)
            if not group:
                continue
            packed = torch.stack([m._local_tensor() for m in group])
            if kind != "none" and live:
                dist.all_reduce(packed, op=dist.ReduceOp.MAX if kind == "max" else dist.ReduceOp.SUM)
                if kind == "mean":
                    packed = packed / dist.get_world_size()
            for m, v in zip(group, packed.unbind(0)):
                m.set_global_tensor(v)

    def reset(self) -> None:
        for m in self._metrics.values():
            m.reset()

    def __getattr__(self, name: str) -> DistributedMetric:
        metrics = self.__dict__.get("_metrics", {})
        if name in metrics:
            return metrics[name]
        raise AttributeError(f"{type(self).__name__} has no metric '{name}'.")
