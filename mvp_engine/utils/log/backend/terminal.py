"""Rank-0 terminal backend (reference: mvp_engine/utils/log/backend/terminal.py:43-179).

Uses ``rich`` when it is importable and plain ``print`` otherwise.
"""

from __future__ import annotations

import inspect
import os
from datetime import datetime
from typing import Mapping, Optional, Union

from ....distributed.utils import is_main_process
from .backend import Backend

try:  # optional pretty printing
    from rich.console import Console

    _CONSOLE = Console(highlight=False)
except Exception:  # pragma: no cover
    _CONSOLE = None


def _caller(depth: int = 3) -> str:
    frame = inspect.currentframe()
    for _ in range(depth):
        if frame is None or frame.f_back is None:
            break
        frame = frame.f_back
    if frame is None:
        return ""
    return f"{os.path.basename(frame.f_code.co_filename)}:{frame.f_lineno}"


class TerminalBackend(Backend):
    def __init__(self, id: str = "", main_process_only: bool = True) -> None:
        self.id = id
        self.enable = (not main_process_only) or is_main_process()

    def _print(self, text: str) -> None:
        if not self.enable:
            return
        if _CONSOLE is not None:
            _CONSOLE.print(text, markup=False)
        else:
            print(text, flush=True)

    def log_metrics(self, metrics: Mapping[str, Union[float, str]], step: int, epoch: Optional[int] = None,
                    total_steps: Optional[int] = None) -> None:
        if not metrics:
            return
        step_str = f"{step}/{total_steps}" if total_steps is not None else str(step)
        fields = []
        for k, v in metrics.items():
            if k == "eta":
                continue
            fields.append(f"{k}: {v:.6g}" if isinstance(v, float) else f"{k}: {v}")
        eta = f" | ETA {metrics['eta']}" if "eta" in metrics else ""
        self._print(f"[{datetime.now():%H:%M:%S}] Step {step_str}{eta} | " + " | ".join(fields))

    def _msg(self, level: str, message: str) -> None:
        self._print(f"[{datetime.now():%H:%M:%S}] {level:<5} {_caller()} {message}")

    def debug(self, message: str) -> None:
        self._msg("DEBUG", message)

    def info(self, message: str) -> None:
        self._msg("INFO", message)

    def warning(self, message: str) -> None:
        self._msg("WARN", message)

    def error(self, message: str) -> None:
        self._msg("ERROR", message)
