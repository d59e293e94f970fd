"""AdamW over the native data-parallel runtime's flat fp32 shards.

One fused kernel per unit does: gradient x (token-normalisation scale) x
(global-norm clip coefficient, computed on device from the all-reduced sum of
squares), decoupled weight decay, the Adam moments, and writes the bf16 copy
of the new weights straight into this rank's slice of the unit's compute
buffer, from where the next step's all-gather starts.  The update rule is
torch.optim.AdamW's single-tensor path, so results match the reference's
optimizer (reference: mvp_engine/kit/optim/__init__.py:11-35).

``param_groups`` behave like any torch optimizer's, so learning-rate
schedulers (e.g. transformers' cosine schedule) drive it unchanged.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from .. import ops
from .fsdp import NativeFSDP


class FlatAdamW(torch.optim.Optimizer):
    def __init__(self, fsdp: NativeFSDP, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.01, **unused: Any) -> None:
        self.fsdp = fsdp
        self.units = [u for u in fsdp.units if u.trainable]
        params = [u.master for u in self.units]
        if not params:
            raise ValueError("No trainable parameters found.")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))
        self._step_count = 0
        self._mvp_native_step = True

    @torch.no_grad()
    def step(self, closure: Optional[Any] = None):
        loss = closure() if closure is not None else None
        f = self.fsdp
        f.finish_grad_sync()
        self._step_count += 1
        g = self.param_groups[0]
        b1, b2 = g["betas"]
        for u in self.units:
            own = u.own_compute_slice(f.rank)
            shadow = own if own.dtype == torch.bfloat16 else None
            ops.adamw_step_(u.master.data, u.grad_shard[: u.shard], u.exp_avg, u.exp_avg_sq, lr=float(g["lr"]), beta1=b1, beta2=b2,
                            eps=float(g["eps"]), weight_decay=float(g["weight_decay"]), step=self._step_count,
                            grad_scale=f._grad_scale, norm_sq=f._norm_sq,
                            max_norm=f._max_norm if f._max_norm is not None else 0.0, p_bf16=shadow)
            if shadow is None:
                own.copy_(u.master.to(own.dtype))
        f.after_optimizer_step()
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        """Gradient buffers are cleared by the runtime right after each update."""

    # ------------------------------------------------------- checkpoints
    def _group_meta(self, fqns: list[str]) -> dict[str, Any]:
        """The param-group entry torch.optim.AdamW of this torch version writes (same keys, so checkpoints
        load into either runtime), with this optimizer's hyper-parameters."""
        g = self.param_groups[0]
        meta = {k: v for k, v in torch.optim.AdamW([torch.zeros(1)]).param_groups[0].items() if k != "params"}
        meta.update(lr=g["lr"], betas=g["betas"], eps=g["eps"], weight_decay=g["weight_decay"], params=fqns)
        if "initial_lr" in g:  # present once a learning-rate scheduler drives the optimizer, as in torch
            meta["initial_lr"] = g["initial_lr"]
        return meta

    def checkpoint_state_dict(self, full: bool = False) -> dict[str, Any]:
        """``{"state": {fqn: {step, exp_avg, exp_avg_sq}}, "param_groups": [...]}`` keyed by HF names."""
        state: dict[str, Any] = {}
        names: list[str] = []
        step = torch.tensor(float(self._step_count))
        for fqns, avg, sq in self.fsdp.optimizer_state_views(full=full):
            for fqn in fqns[:1]:
                state[fqn] = {"step": step.clone(), "exp_avg": avg, "exp_avg_sq": sq}
                names.append(fqn)
        return {"state": state, "param_groups": [self._group_meta(names)]}

    def load_checkpoint_state_dict(self, sd: dict[str, Any], full: bool = False) -> None:
        state = sd.get("state", {})
        self.fsdp.load_optimizer_views(state)
        steps = [v["step"] for v in state.values() if isinstance(v, dict) and "step" in v]
        if steps:
            self._step_count = int(float(steps[0]))
        groups = sd.get("param_groups") or []
        if groups:
            for k in ("lr", "betas", "eps", "weight_decay", "initial_lr"):
                if k in groups[0]:
                    self.param_groups[0][k] = groups[0][k]
