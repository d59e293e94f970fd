"""Token-normalised loss accounting (reference: mvp_engine/kit/loss/token_loss.py:17-311).

Each micro-batch backpropagates ``sum(per-token loss) / backward_divisor`` with
a fixed divisor; once per optimizer step ``reduce_window`` all-reduces the
token counts and the loss sum over the data-parallel group and returns
``gradient_scale = divisor * dp_world / global_effective_tokens``, the factor
that turns the accumulated gradients into the gradient of the mean loss over
every supervised token of the step.  ``rescale_gradients`` applies it; with
the native data-parallel runtime it is folded into the optimizer update
instead of a separate pass over the gradients.
"""

from __future__ import annotations

import inspect
from dataclasses import dataclass
from types import MethodType
from typing import Any, Iterable, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .loss import LossGuard


@dataclass(frozen=True)
class TokenLossStats:
    global_total_tokens: int
    global_effective_tokens: int
    global_loss_sum: float
    backward_divisor: int
    gradient_scale: float


class PerTokenLossGuard(LossGuard):
    """Spike guard on the dp-global mean per-token loss of a micro-batch."""

    def __init__(self, *, spike_multiplier, window_size, min_history, group=None, group_world_size=None):
        super().__init__(spike_multiplier=spike_multiplier, window_size=window_size, min_history=min_history)
        self.group = group
        self.group_world_size = group_world_size

    def check(self, loss_sum, token_count: int, *, step: int, device: torch.device) -> bool:  # type: ignore[override]
        if self.spike_multiplier is None:
            return False
        s = (loss_sum.detach().to(device=device, dtype=torch.float32) if isinstance(loss_sum, torch.Tensor)
             else torch.tensor(float(loss_sum), device=device, dtype=torch.float32))
        n = torch.tensor(int(token_count), device=device, dtype=torch.int64)
        if (self.group_world_size is None or self.group_world_size > 1) and dist.is_available() and dist.is_initialized():
            dist.all_reduce(s, group=self.group)
            dist.all_reduce(n, group=self.group)
        total = int(n.item())
        if total <= 0:
            return False
        return super().check(s / n, step=step, token_count=total)


class TokenNormedLossKit:
    def __init__(self, *, device: torch.device, dp_world_size: int, dp_group=None,
                 loss_guard: Optional[PerTokenLossGuard] = None, loss_sum_group=None) -> None:
        """``loss_sum_group``: ranks that each hold part of every sample's per-token losses while
        counting the sample's tokens in full (sequence-parallel tensor ranks); loss sums are
        additionally summed over it."""
        self.device = device
        self.dp_world_size = int(dp_world_size)
        self.dp_group = dp_group
        self.loss_sum_group = loss_sum_group
        self.loss_guard = loss_guard
        self.reset()

    def apply_chunked_token_loss_patch(self, model: torch.nn.Module, *, chunk_size: int = 4096,
                                       output_cls: type | None = None) -> torch.nn.Module:
        return apply_chunked_token_loss_patch(model, chunk_size=chunk_size, output_cls=output_cls)

    def build_loss_guard(self, *, spike_multiplier, window_size: int, min_history: int, group=None,
                         group_world_size=None) -> PerTokenLossGuard:
        self.loss_guard = PerTokenLossGuard(spike_multiplier=spike_multiplier, window_size=window_size,
                                            min_history=min_history,
                                            group=self.dp_group if group is None else group,
                                            group_world_size=self.dp_world_size if group_world_size is None
                                            else group_world_size)
        return self.loss_guard

    def guard_loss(self, loss_sum, token_count: int, *, step: int = 0) -> bool:
        if self.loss_guard is None:
            return True
        return not self.loss_guard.check(loss_sum, int(token_count), step=step, device=self.device)

    def accumulate_microbatch(self, *, loss_sum: torch.Tensor, effective_tokens: int, total_tokens: int,
                              backward_divisor: int) -> torch.Tensor:
        if backward_divisor <= 0:
            raise ValueError("backward_divisor must be positive.")
        if effective_tokens < 0 or total_tokens < 0:
            raise ValueError("Token counts must be non-negative.")
        if self._backward_divisor is None:
            self._backward_divisor = int(backward_divisor)
        elif self._backward_divisor != int(backward_divisor):
            raise ValueError("backward_divisor must stay fixed within one accumulation window.")
        self._total_tokens += int(total_tokens)
        self._effective_tokens += int(effective_tokens)
        d = loss_sum.detach().to(device=self.device, dtype=torch.float32)
        self._loss_sum = d if self._loss_sum is None else self._loss_sum + d
        return loss_sum / float(backward_divisor)

    def reduce_window(self) -> TokenLossStats:
        if self._backward_divisor is None or self._loss_sum is None:
            raise RuntimeError("No token loss has been accumulated.")
        counts = torch.tensor([self._total_tokens, self._effective_tokens], device=self.device, dtype=torch.int64)
        loss_sum = self._loss_sum.clone().reshape(())
        if dist.is_available() and dist.is_initialized() and self.dp_world_size > 1:
            dist.all_reduce(counts, group=self.dp_group)
            dist.all_reduce(loss_sum, group=self.dp_group)
        if self.loss_sum_group is not None:
            dist.all_reduce(loss_sum, group=self.loss_sum_group)
        c = counts.tolist()
        if c[1] <= 0:
            raise ValueError("Accumulation window must contain at least one supervised token.")
        scale = float(self._backward_divisor) * float(self.dp_world_size) / float(c[1])
        return TokenLossStats(global_total_tokens=int(c[0]), global_effective_tokens=int(c[1]),
                              global_loss_sum=float(loss_sum.item()), backward_divisor=int(self._backward_divisor),
                              gradient_scale=scale)

    def rescale_gradients(self, parameters: Iterable[torch.nn.Parameter] | torch.nn.Module,
                          stats: TokenLossStats) -> None:
        """Multiply gradients by ``stats.gradient_scale`` (folded into the update for native models)."""
        target = parameters
        native = getattr(target, "scale_gradients_", None)
        if callable(native):
            native(stats.gradient_scale)
            return
        with torch.no_grad():
            for p in target:
                if p.grad is not None:
                    p.grad.mul_(stats.gradient_scale)

    def reset(self) -> None:
        self._total_tokens = 0
        self._effective_tokens = 0
        self._loss_sum: Optional[torch.Tensor] = None
        self._backward_divisor: Optional[int] = None


def apply_chunked_token_loss_patch(model: torch.nn.Module, *, chunk_size: int = 4096,
                                   output_cls: type | None = None) -> torch.nn.Module:
    """Make a causal LM return the unreduced per-token loss, computing logits in chunks.

    Models of this engine already do this natively (their forward runs the
    fused linear + cross-entropy kernels and never materialises full logits);
    for them the patch only sets the chunk size.  Any other causal LM exposing
    ``.model`` and ``.lm_head`` gets a wrapped forward with the reference's
    semantics: labels shifted by one with -100 padding, ``F.linear`` +
    ``F.cross_entropy(reduction="none")`` per chunk, ``logits=None``.
    """
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive.")
    if hasattr(model, "loss_chunk_size"):
        model.loss_chunk_size = int(chunk_size)
        return model
    if not hasattr(model, "model") or not hasattr(model, "lm_head"):
        raise ValueError("Chunked token loss patch requires the model to expose `.model` and `.lm_head`.")
    outer = inspect.signature(model.forward)
    inner = inspect.signature(model.model.forward)
    inner_kwargs = any(p.kind == p.VAR_KEYWORD for p in inner.parameters.values())
    inner_names = set(inner.parameters)
    bias = getattr(model.lm_head, "bias", None)

    def forward(self, *args: Any, **kwargs: Any):
        if args:
            bound = outer.bind_partial(*args, **kwargs)
            bound.apply_defaults()
            kw = dict(bound.arguments)
            kw.update(kw.pop("kwargs", {}))
        else:
            kw = dict(kwargs)
        labels = kw.pop("labels", None)
        keep = kw.pop("logits_to_keep", 0)
        if not inner_kwargs:
            kw = {k: v for k, v in kw.items() if k in inner_names}
        out = self.model(**kw)
        h = out[0]
        sl = slice(-keep, None) if isinstance(keep, int) else keep
        h = h[:, sl, :] if h.dim() == 3 else h[sl, :]
        if labels is None:
            res = {"loss": None, "logits": self.lm_head(h)}
        else:
            lab = F.pad(labels, (0, 1), value=-100)[..., 1:].contiguous()
            lab = lab[:, sl] if lab.dim() == 2 else lab[sl]
            hf, lf = h.reshape(-1, h.size(-1)), lab.reshape(-1)
            parts = [F.cross_entropy(F.linear(hf[s:s + chunk_size], self.lm_head.weight, bias), lf[s:s + chunk_size],
                                     ignore_index=-100, reduction="none") for s in range(0, hf.size(0), chunk_size)]
            res = {"loss": torch.cat(parts), "logits": None}
        if output_cls is not None:
            names = set(inspect.signature(output_cls).parameters)
            return output_cls(**{k: v for k, v in res.items() if k in names})
        return res

    forward.__signature__ = outer
    model.forward = MethodType(forward, model)
    return model
