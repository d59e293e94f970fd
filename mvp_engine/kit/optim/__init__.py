"""Optimizer / scheduler construction (reference: mvp_engine/kit/optim/__init__.py:11-50).

``build_optimizer(model, "AdamW", lr, wd)`` returns the fused flat-shard AdamW
when ``model`` is the native data-parallel runtime (same update rule as
``torch.optim.AdamW``), and ``getattr(torch.optim, name)`` over the trainable
parameters otherwise.
"""

from __future__ import annotations

import math
from typing import Any

import torch


class OptimKit:
    def build_optimizer(self, model: torch.nn.Module, optimizer: str, lr: float, weight_decay: float,
                        **kwargs: Any) -> torch.optim.Optimizer:
        from ...parallel.fsdp import NativeFSDP

        base = getattr(model, "_orig_mod", model)
        if isinstance(base, NativeFSDP):
            if optimizer == "AdamW" and not kwargs.get("amsgrad", False):
                from ...parallel.optim import FlatAdamW

                return FlatAdamW(base, lr=lr, weight_decay=weight_decay, **kwargs)
            assert hasattr(torch.optim, optimizer), f"Optimizer '{optimizer}' not found in torch.optim."
            opt = getattr(torch.optim, optimizer)(list(base.shard_params), lr=lr, weight_decay=weight_decay, **kwargs)
            return base.attach_optimizer(opt)
        params = [p for p in model.parameters() if p.requires_grad]
        if not params:
            raise ValueError("No trainable parameters found.")
        assert hasattr(torch.optim, optimizer), f"Optimizer '{optimizer}' not found in torch.optim."
        return getattr(torch.optim, optimizer)(params, lr=lr, weight_decay=weight_decay, **kwargs)

    def build_lr_scheduler(self, optimizer: torch.optim.Optimizer, lr_scheduler: str, **kwargs: Any):
        """transformers' ``get_scheduler`` when importable, else the same cosine/linear/constant rules."""
        try:
            from transformers import get_scheduler

            return get_scheduler(name=lr_scheduler, optimizer=optimizer, **kwargs)
        except ImportError:  # pragma: no cover
            return build_builtin_scheduler(optimizer, lr_scheduler, **kwargs)


def build_builtin_scheduler(optimizer, name: str, num_warmup_steps: int = 0, num_training_steps: int = 1, **_: Any):
    def lam(step: int) -> float:
        if step < num_warmup_steps:
            return step / max(1, num_warmup_steps)
        if name == "constant" or name == "constant_with_warmup":
            return 1.0
        prog = (step - num_warmup_steps) / max(1, num_training_steps - num_warmup_steps)
        if name == "linear":
            return max(0.0, 1.0 - prog)
        return max(0.0, 0.5 * (1.0 + math.cos(math.pi * prog)))

    return torch.optim.lr_scheduler.LambdaLR(optimizer, lam)
