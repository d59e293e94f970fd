"""Weights & Biases backend; disabled unless ``wandb`` imports and a key or mode is set
(reference: mvp_engine/utils/log/backend/wandb.py:24-108)."""

from __future__ import annotations

import os
from pathlib import Path
from typing import Mapping, Optional, Union

from ....distributed.utils import is_main_process
from .backend import Backend


class WandbBackend(Backend):
    def __init__(self, id: str, project: str, path: Union[str, Path], main_process_only: bool = True) -> None:
        self.run = None
        if main_process_only and not is_main_process():
            return
        if not (os.environ.get("WANDB_API_KEY") or os.environ.get("WANDB_MODE")):
            return
        try:
            import wandb  # type: ignore
        except Exception:
            return
        Path(path).mkdir(parents=True, exist_ok=True)
        self.run = wandb.init(project=project, name=id, id=id, dir=str(path), resume="allow")

    def log_config(self, config: dict) -> None:
        if self.run is not None:
            self.run.config.update(config, allow_val_change=True)

    def log_metrics(self, metrics: Mapping[str, Union[float, str]], step: int, epoch: Optional[int] = None,
                    total_steps: Optional[int] = None) -> None:
        if self.run is not None:
            self.run.log({k: v for k, v in metrics.items() if not isinstance(v, str)}, step=step)

    def destroy(self) -> None:
        if self.run is not None:
            self.run.finish()
            self.run = None
