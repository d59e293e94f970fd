"""Weights & Biases backend; disabled unless ``wandb`` imports and a key or mode is set
(reference: mvp_engine/utils/log/backend/wandb.py:24-108)."""

from __future__ import annotations

import os
from pathlib import Path
from typing import Mapping, Optional, Union

from ....distributed.utils import is_main_process
from .backend import Backend


class WandbBackend(Backend):
    def __init__(self, id: str, project: str, entity: Optional[str] = None, config: Optional[Mapping] = None,
                 path: Optional[Union[str, Path]] = None, main_process_only: bool = True) -> None:
        """``entity`` / ``config`` go to ``wandb.init`` (an OmegaConf config is converted to plain dicts).
        Nothing is started on non-main ranks, without ``wandb``, or without credentials / a ``WANDB_MODE``
        (no interactive login)."""
        self.run = None
        if main_process_only and not is_main_process():
            return
        if not (os.environ.get("WANDB_API_KEY") or os.environ.get("WANDB_MODE")):
            return
        try:
            import wandb  # type: ignore
        except Exception:
            return
        if config is not None and not isinstance(config, dict):
            try:
                from omegaconf import OmegaConf

                config = OmegaConf.to_container(config, resolve=True)
            except ImportError:
                config = dict(config)
        if path is not None:
            Path(path).mkdir(parents=True, exist_ok=True)
        self.run = wandb.init(project=project, entity=entity, name=id, id=id, config=config,
                              dir=str(path) if path is not None else None, resume="allow")

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
