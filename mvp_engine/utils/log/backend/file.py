"""Rank-0 file backend: ``log_<id>.log`` and ``config_<id>.yaml`` in the run directory.

The line format (``date | id | ETA x | Step s/total || key: value | ...``) is
the one the reference's run-summary tooling parses
(reference: mvp_engine/utils/log/backend/file.py:19-109).
"""

from __future__ import annotations

from datetime import datetime
from pathlib import Path
from typing import Mapping, Optional, Union

import yaml

from ....distributed.utils import is_main_process
from .backend import Backend


class FileBackend(Backend):
    def __init__(self, id: str, path: Union[str, Path], main_process_only: bool = True) -> None:
        self.id = id
        self.path = Path(path)
        self.enable = (not main_process_only) or is_main_process()
        self.log_file = None
        if self.enable:
            self.path.mkdir(parents=True, exist_ok=True)
            self.log_file = open(self.path / f"log_{id}.log", "w")

    @staticmethod
    def _now() -> str:
        return datetime.now().strftime("%Y-%m-%d %H:%M:%S")

    def log_config(self, config: dict) -> None:
        if self.enable:
            with open(self.path / f"config_{self.id}.yaml", "w") as f:
                yaml.safe_dump(config, f, default_flow_style=False, allow_unicode=True, sort_keys=False)

    def log_metrics(self, metrics: Mapping[str, Union[float, str]], step: int, epoch: Optional[int] = None,
                    total_steps: Optional[int] = None) -> None:
        if not self.enable or self.log_file is None or not metrics:
            return
        parts = [self._now(), self.id]
        if "eta" in metrics:
            parts.append(f"ETA {metrics['eta']}")
        head = " | ".join(parts)
        epoch_str = f"Epoch {epoch} - " if epoch is not None else ""
        step_str = f"{step:>8}/{total_steps}" if total_steps is not None else f"{step:>8}"
        body = "".join(f"{k}: {v} | " for k, v in metrics.items() if k != "eta")
        self.log_file.write(f"{head} | {epoch_str}Step {step_str} || {body}\n")
        self.log_file.flush()

    def _msg(self, level: str, message: str) -> None:
        if self.enable and self.log_file is not None:
            self.log_file.write(f"{self._now()} | {self.id} | {level:<5} | {message}\n")
            self.log_file.flush()

    def debug(self, message: str) -> None:
        self._msg("DEBUG", message)

    def info(self, message: str) -> None:
        self._msg("INFO", message)

    def warning(self, message: str) -> None:
        self._msg("WARN", message)

    def error(self, message: str) -> None:
        self._msg("ERROR", message)

    def destroy(self) -> None:
        if self.log_file is not None:
            self.log_file.close()
            self.log_file = None
