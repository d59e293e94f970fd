"""Log backend interface (reference: mvp_engine/utils/log/backend/backend.py:4-49)."""

from __future__ import annotations

from typing import Mapping, Optional, Union


class Backend:
    """Receives configs, aggregated metrics and messages from the Logger."""

    def log_config(self, config: dict) -> None:
        pass

    def log_metrics(
        self,
        metrics: Mapping[str, Union[float, str]],
        step: int,
        epoch: Optional[int] = None,
        total_steps: Optional[int] = None,
    ) -> None:
        pass

    def destroy(self) -> None:
        pass

    def info(self, message: str) -> None:
        pass

    def debug(self, message: str) -> None:
        pass

    def warning(self, message: str) -> None:
        pass

    def error(self, message: str) -> None:
        pass
