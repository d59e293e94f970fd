#!/usr/bin/env python3
"""Summarise one run directory of this engine as JSON.

A run directory (``<project.dir>/<run_id>/``) holds what the engine wrote: the file backend's
``log_<run_id>.log`` (metric lines ``date | id | [ETA x |] Step s/total || key: value | ...`` and message
lines ``date | id | LEVEL | text``), ``config_<run_id>.yaml``, and ``checkpoints/<policy>_<n>/`` whose
``COMPLETE`` marker says the checkpoint was fully written (its content is the optimizer step).

The summary has four parts:

* ``run``: the config keys a reader needs first (engine, model, batch, parallel layout, optimizer, loop);
* ``metrics``: per logged key, the count, first / last value and step, min, max, mean, the mean of the
  last ``--window`` points and those points themselves;
* ``health``: loss trend (mean of the first window against the last), non-finite values seen, message
  counts per level and the last warnings / errors, and the step range covered;
* ``checkpoints``: every checkpoint directory with its completeness, and the newest complete one (what
  ``resume: latest`` would load).

Usage::

    python skills/experiment/experiment-analysis/scripts/summarize_run.py --run-dir outputs/<run_id> \
        [--output summary.json] [--window 5] [--with-config]
"""

from __future__ import annotations

import argparse
import json
import math
import re
import sys
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Optional

try:
    import yaml
except ImportError:  # pragma: no cover - yaml ships with the engine's dependencies
    yaml = None

_METRIC_LINE = re.compile(r"\|\s*(?:Epoch (?P<epoch>\d+) - )?Step\s+(?P<step>\d+)(?:/(?P<total>\d+))?\s*\|\|(?P<body>.*)$")
_MESSAGE_LINE = re.compile(r"^\S+ \S+ \| [^|]+ \| (?P<level>DEBUG|INFO|WARN|ERROR)\s*\| (?P<text>.*)$")
_RUN_KEYS = (
    "engine", "runtime.run_id", "runtime.git_info", "runtime.world_size", "project.name",
    "model.pretrained_model_name_or_path", "data.max_seq_len", "data.batch_size", "optim.global_batch_size",
    "optim.gradient_accumulation_steps", "optim.lr", "optim.mixed_precision", "optim.clip_grad_norm",
    "parallel.mesh", "parallel.backend_kwargs.impl", "loop.policy", "loop.total_steps", "checkpoint.interval",
    "checkpoint.keep_n", "resume",
)
_LOSS_KEYS = ("train/loss", "loss")


def _value(text: str) -> Any:
    text = text.strip()
    for cast in (int, float):
        try:
            return cast(text)
        except ValueError:
            pass
    low = text.lower()
    if low in ("nan", "inf", "-inf"):
        return float(low)
    return text


def _dotted(tree: Any, key: str) -> Any:
    for part in key.split("."):
        if not isinstance(tree, dict) or part not in tree:
            return None
        tree = tree[part]
    return tree


@dataclass
class Series:
    points: list[tuple[int, float]] = field(default_factory=list)
    non_finite: int = 0

    def add(self, step: int, v: float) -> None:
        if not math.isfinite(v):
            self.non_finite += 1
            return
        self.points.append((step, v))

    def describe(self, window: int) -> dict[str, Any]:
        if not self.points:
            return {"count": 0, "non_finite": self.non_finite}
        vals = [v for _, v in self.points]
        tail = self.points[-window:]
        return {
            "count": len(vals), "non_finite": self.non_finite,
            "first": {"step": self.points[0][0], "value": vals[0]},
            "last": {"step": self.points[-1][0], "value": vals[-1]},
            "min": min(vals), "max": max(vals), "mean": sum(vals) / len(vals),
            "window_mean": sum(v for _, v in tail) / len(tail),
            "tail": [{"step": s, "value": v} for s, v in tail],
        }


@dataclass
class LogScan:
    series: dict[str, Series] = field(default_factory=dict)
    text_values: dict[str, str] = field(default_factory=dict)
    levels: dict[str, int] = field(default_factory=dict)
    problems: list[str] = field(default_factory=list)
    steps: list[int] = field(default_factory=list)
    total_steps: Optional[int] = None

    def feed(self, line: str) -> None:
        line = line.rstrip("\n")
        m = _METRIC_LINE.search(line)
        if m:
            step = int(m["step"])
            self.steps.append(step)
            if m["total"]:
                self.total_steps = int(m["total"])
            for item in m["body"].split(" | "):
                key, sep, raw = item.partition(": ")
                key = key.strip()
                if not sep or not key:
                    continue
                val = _value(raw)
                if isinstance(val, (int, float)):
                    self.series.setdefault(key, Series()).add(step, float(val))
                else:
                    self.text_values[key] = val
            return
        m = _MESSAGE_LINE.match(line)
        if m:
            self.levels[m["level"]] = self.levels.get(m["level"], 0) + 1
            if m["level"] in ("WARN", "ERROR"):
                self.problems.append(f"{m['level']}: {m['text']}")


def _scan_log(path: Optional[Path]) -> LogScan:
    scan = LogScan()
    if path is not None:
        with open(path, encoding="utf-8", errors="replace") as f:
            for line in f:
                scan.feed(line)
    return scan


def _checkpoints(run_dir: Path) -> dict[str, Any]:
    root = run_dir / "checkpoints"
    found = []
    if root.is_dir():
        for p in root.iterdir():
            head, _, tail = p.name.rpartition("_")
            if not (p.is_dir() and head and tail.isdigit()):
                continue
            marker = p / "COMPLETE"
            step = None
            if marker.is_file():
                text = marker.read_text().strip()
                step = int(text) if text.isdigit() else None
            found.append({"name": p.name, "index": int(tail), "complete": marker.is_file(), "step": step,
                          "hf_export": (p / "hf_model").is_dir()})
    found.sort(key=lambda c: c["index"])
    complete = [c for c in found if c["complete"]]
    return {"directories": found, "latest_complete": complete[-1]["name"] if complete else None,
            "incomplete": [c["name"] for c in found if not c["complete"]]}


def _first(run_dir: Path, pattern: str) -> Optional[Path]:
    hits = sorted(run_dir.glob(pattern), key=lambda p: p.stat().st_mtime)
    return hits[-1] if hits else None


def summarize(run_dir: Path, *, window: int = 5, with_config: bool = False) -> dict[str, Any]:
    run_dir = Path(run_dir)
    if not run_dir.is_dir():
        raise FileNotFoundError(f"no run directory at {run_dir}")
    log_path = _first(run_dir, "log_*.log")
    cfg_path = _first(run_dir, "config_*.yaml")
    config: dict[str, Any] = {}
    if cfg_path is not None and yaml is not None:
        config = yaml.safe_load(cfg_path.read_text()) or {}
    scan = _scan_log(log_path)
    metrics = {k: s.describe(window) for k, s in sorted(scan.series.items())}
    loss_key = next((k for k in _LOSS_KEYS if k in scan.series and scan.series[k].points), None)
    trend = None
    if loss_key:
        vals = [v for _, v in scan.series[loss_key].points]
        head, tail = vals[:window], vals[-window:]
        trend = {"key": loss_key, "first_window_mean": sum(head) / len(head),
                 "last_window_mean": sum(tail) / len(tail),
                 "decreased": sum(tail) / len(tail) < sum(head) / len(head)}
    out = {
        "run_dir": str(run_dir.resolve()),
        "files": {"log": str(log_path) if log_path else None, "config": str(cfg_path) if cfg_path else None},
        "run": {k: _dotted(config, k) for k in _RUN_KEYS if _dotted(config, k) is not None},
        "metrics": metrics,
        "text_metrics": scan.text_values,
        "health": {
            "steps_logged": len(scan.steps),
            "step_range": [min(scan.steps), max(scan.steps)] if scan.steps else None,
            "total_steps": scan.total_steps,
            "finished": bool(scan.steps) and scan.total_steps is not None and max(scan.steps) >= scan.total_steps,
            "loss_trend": trend,
            "non_finite": {k: s.non_finite for k, s in scan.series.items() if s.non_finite},
            "messages": scan.levels,
            "last_problems": scan.problems[-5:],
        },
        "checkpoints": _checkpoints(run_dir),
    }
    if with_config:
        out["config"] = config
    return out


def main(argv: Optional[list[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--run-dir", type=Path, required=True, help="<project.dir>/<run_id> of the run")
    ap.add_argument("--output", type=Path, default=None, help="write the JSON here instead of stdout")
    ap.add_argument("--window", type=int, default=5, help="points per metric in the tail / trend windows")
    ap.add_argument("--with-config", action="store_true", help="include the whole config")
    args = ap.parse_args(argv)
    summary = summarize(args.run_dir, window=max(1, args.window), with_config=args.with_config)
    text = json.dumps(summary, indent=2, sort_keys=False, default=str)
    if args.output:
        args.output.write_text(text + "\n")
    else:
        sys.stdout.write(text + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
