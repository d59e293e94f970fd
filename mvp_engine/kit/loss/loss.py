"""Scalar loss helpers and the loss-spike guard (reference: mvp_engine/kit/loss/loss.py:14-95)."""

from __future__ import annotations

from collections import deque
from typing import Any, Optional

import torch

from ...utils.log import simple_info


class LossGuard:
    """Skip a micro-batch whose loss exceeds ``multiplier`` x the mean of recent accepted losses.

    The first ``min_history`` losses only fill the window.  A skipped loss is
    not added to the history.
    """

    def __init__(self, *, spike_multiplier: Optional[float], window_size: int, min_history: int) -> None:
        self.spike_multiplier = spike_multiplier
        self.min_history = int(min_history)
        self.loss_history: deque[float] = deque(maxlen=int(window_size))

    def check(self, loss: Any, *, step: int, token_count: Optional[int] = None) -> bool:
        if self.spike_multiplier is None:
            return False
        cur = float(loss.detach().item()) if isinstance(loss, torch.Tensor) else float(loss)
        if len(self.loss_history) < self.min_history:
            self.loss_history.append(cur)
            return False
        base = sum(self.loss_history) / len(self.loss_history)
        if cur > base * float(self.spike_multiplier):
            extra = f", micro_tokens={token_count}" if token_count is not None else ""
            simple_info(f"Loss spike skip at step {step}: micro_loss={cur:.4f}, baseline_loss={base:.4f}, "
                        f"history_size={len(self.loss_history)}, loss_factor={cur / base if base > 0 else float('inf'):.2f}, "
                        f"spike_multiplier={self.spike_multiplier}{extra}", level="warning")
            return True
        self.loss_history.append(cur)
        return False


class LossKit:
    def __init__(self, loss_guard: Optional[LossGuard] = None) -> None:
        self.loss_guard = loss_guard

    def build_loss_guard(self, *, spike_multiplier: Optional[float], window_size: int, min_history: int) -> LossGuard:
        self.loss_guard = LossGuard(spike_multiplier=spike_multiplier, window_size=window_size,
                                    min_history=min_history)
        return self.loss_guard

    def guard_loss(self, loss: Any, *, step: int = 0) -> bool:
        """True when ``loss`` should take part in backward."""
        return True if self.loss_guard is None else not self.loss_guard.check(loss, step=step)
