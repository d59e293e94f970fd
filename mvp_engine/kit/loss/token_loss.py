"""Token-normalised loss: the gradient of the mean loss over every supervised token of a step.

Public API of the reference's ``mvp_engine/kit/loss/token_loss.py:17-311``: ``TokenNormedLossKit``
(``accumulate_microbatch`` / ``reduce_window`` / ``rescale_gradients`` / ``guard_loss``),
``TokenLossStats``, ``PerTokenLossGuard`` and ``apply_chunked_token_loss_patch``.

How it works here.  Every micro-batch backpropagates ``sum(per-token loss) / divisor`` with a
divisor that is fixed for the step, so backward can start before the step's global token
count is known.  The kit keeps the step's running totals in a :class:`_Window`; at the end
of the step ``reduce_window`` sums ``[all tokens, supervised tokens, loss sum]`` over the
data-parallel group with ONE all-reduce of a float64 vector (exact for counts below 2^53),
and returns ``gradient_scale = divisor * dp_world / global supervised tokens``: the factor
that turns the accumulated gradients into the gradient of the step's mean token loss.
Models of this engine's native runtime take that factor inside the optimizer update
(``scale_gradients_``), so no extra pass over the gradients is made.
"""

from __future__ import annotations

import inspect
from dataclasses import dataclass
from types import MethodType
from typing import Any, Iterable, Optional, Union

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


def _dist_live() -> bool:
    return dist.is_available() and dist.is_initialized()


def _as_f64(x: Union[torch.Tensor, float], device: torch.device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.detach().to(device=device, dtype=torch.float64).reshape(())
    return torch.tensor(float(x), device=device, dtype=torch.float64)


class PerTokenLossGuard(LossGuard):
    """Spike guard on the group-wide mean per-token loss of one micro-batch.

    ``check`` reduces ``(loss sum, token count)`` over ``group`` in one all-reduce, so every rank
    takes the same decision."""

    def __init__(self, *, spike_multiplier, window_size, min_history, group=None, group_world_size=None):
        super().__init__(spike_multiplier=spike_multiplier, window_size=window_size, min_history=min_history)
        self.group = group
        self.group_world_size = group_world_size

    def check(self, loss_sum, token_count: int, *, step: int, device: torch.device) -> bool:  # type: ignore[override]
        if self.spike_multiplier is None:
            return False
        pair = torch.stack([_as_f64(loss_sum, device), _as_f64(float(token_count), device)])
        if _dist_live() and (self.group_world_size is None or self.group_world_size > 1):
            dist.all_reduce(pair, group=self.group)
        total_loss, tokens = pair.tolist()
        if tokens <= 0:
            return False
        return super().check(total_loss / tokens, step=step, token_count=int(tokens))


@dataclass
class _Window:
    """Running totals of one optimizer step on this rank."""

    divisor: Optional[int] = None
    all_tokens: int = 0
    supervised_tokens: int = 0
    loss_sum: Optional[torch.Tensor] = None

    def add(self, loss_sum: torch.Tensor, supervised: int, total: int, divisor: int) -> None:
        if self.divisor is None:
            self.divisor = divisor
        elif self.divisor != divisor:
            raise ValueError("backward_divisor must stay fixed within one accumulation window.")
        self.all_tokens += total
        self.supervised_tokens += supervised
        self.loss_sum = loss_sum if self.loss_sum is None else self.loss_sum + loss_sum


class TokenNormedLossKit:
    def __init__(self, *, device: torch.device, dp_world_size: int, dp_group=None,
                 loss_guard: Optional[PerTokenLossGuard] = None, loss_sum_group=None) -> None:
        """``loss_sum_group``: ranks that each hold part of every sample's per-token losses while
        counting the sample's tokens in full (sequence-parallel tensor ranks); their loss sums are
        added as well."""
        self.device = device
        self.dp_world_size = int(dp_world_size)
        self.dp_group = dp_group
        self.loss_sum_group = loss_sum_group
        self.loss_guard = loss_guard
        self._window = _Window()

    def apply_chunked_token_loss_patch(self, model: torch.nn.Module, *, chunk_size: int = 4096,
                                       output_cls: Optional[type] = None) -> torch.nn.Module:
        return apply_chunked_token_loss_patch(model, chunk_size=chunk_size, output_cls=output_cls)

    def build_loss_guard(self, *, spike_multiplier, window_size: int, min_history: int, group=None,
                         group_world_size=None) -> PerTokenLossGuard:
        if group is None:
            group = self.dp_group
        if group_world_size is None:
            group_world_size = self.dp_world_size
        self.loss_guard = PerTokenLossGuard(spike_multiplier=spike_multiplier, window_size=window_size,
                                            min_history=min_history, group=group, group_world_size=group_world_size)
        return self.loss_guard

    def guard_loss(self, loss_sum, token_count: int, *, step: int = 0) -> bool:
        """True when the micro-batch should take part in backward."""
        guard = self.loss_guard
        return guard is None or not guard.check(loss_sum, int(token_count), step=step, device=self.device)

    def accumulate_microbatch(self, *, loss_sum: torch.Tensor, effective_tokens: int, total_tokens: int,
                              backward_divisor: int) -> torch.Tensor:
        """Record one micro-batch and return the loss to backpropagate (``loss_sum / divisor``)."""
        if backward_divisor <= 0:
            raise ValueError("backward_divisor must be positive.")
        if min(effective_tokens, total_tokens) < 0:
            raise ValueError("Token counts must be non-negative.")
        self._window.add(loss_sum.detach().to(device=self.device, dtype=torch.float32), int(effective_tokens),
                         int(total_tokens), int(backward_divisor))
        return loss_sum / float(backward_divisor)

    def reduce_window(self) -> TokenLossStats:
        w = self._window
        if w.divisor is None or w.loss_sum is None:
            raise RuntimeError("No token loss has been accumulated.")
        totals = torch.stack([_as_f64(float(w.all_tokens), self.device),
                              _as_f64(float(w.supervised_tokens), self.device), _as_f64(w.loss_sum, self.device)])
        if _dist_live() and self.dp_world_size > 1:
            dist.all_reduce(totals, group=self.dp_group)
        if self.loss_sum_group is not None:
            # only the loss sum is split over these ranks; their token counts are already whole
            part = totals[2:].clone()
            dist.all_reduce(part, group=self.loss_sum_group)
            totals[2:] = part
        all_tokens, supervised, loss = totals.tolist()
        if supervised <= 0:
            raise ValueError("Accumulation window must contain at least one supervised token.")
        return TokenLossStats(global_total_tokens=int(all_tokens), global_effective_tokens=int(supervised),
                              global_loss_sum=float(loss), backward_divisor=int(w.divisor),
                              gradient_scale=float(w.divisor) * self.dp_world_size / supervised)

    def rescale_gradients(self, parameters: Union[Iterable[torch.nn.Parameter], torch.nn.Module],
                          stats: TokenLossStats) -> None:
        """Multiply the accumulated gradients by ``stats.gradient_scale``.

        A native-runtime model (``scale_gradients_``) folds the factor into its optimizer update."""
        fold = getattr(parameters, "scale_gradients_", None)
        if callable(fold):
            fold(stats.gradient_scale)
            return
        grads = [p.grad for p in parameters if p.grad is not None]
        if grads:
            torch._foreach_mul_(grads, stats.gradient_scale)

    def reset(self) -> None:
        self._window = _Window()


class _ChunkedLossForward:
    """Replacement ``forward`` for a causal LM: per-token CE from chunked logits, ``logits=None``.

    Labels are shifted left by one (last position gets -100); each chunk of ``chunk_size`` rows
    runs ``lm_head`` and ``F.cross_entropy(reduction="none")``, so full logits never exist."""

    def __init__(self, model: torch.nn.Module, chunk_size: int, output_cls: Optional[type]) -> None:
        self.outer_sig = inspect.signature(model.forward)
        inner_sig = inspect.signature(model.model.forward)
        self.inner_takes_any = any(p.kind == p.VAR_KEYWORD for p in inner_sig.parameters.values())
        self.inner_names = frozenset(inner_sig.parameters)
        self.chunk = int(chunk_size)
        self.output_fields = frozenset(inspect.signature(output_cls).parameters) if output_cls else None
        self.output_cls = output_cls

    def _kwargs(self, args: tuple, kwargs: dict) -> dict:
        if not args:
            return dict(kwargs)
        bound = self.outer_sig.bind_partial(*args, **kwargs)
        bound.apply_defaults()
        merged = dict(bound.arguments)
        merged.update(merged.pop("kwargs", {}))
        return merged

    def _token_losses(self, lm: torch.nn.Module, h: torch.Tensor, labels: torch.Tensor, keep) -> torch.Tensor:
        sel = slice(-keep, None) if isinstance(keep, int) else keep
        target = F.pad(labels, (0, 1), value=-100)[..., 1:]
        target = (target[:, sel] if target.dim() == 2 else target[sel]).reshape(-1)
        rows = h.reshape(-1, h.size(-1))
        bias = getattr(lm.lm_head, "bias", None)
        losses = []
        for lo in range(0, rows.size(0), self.chunk):
            logits = F.linear(rows[lo:lo + self.chunk], lm.lm_head.weight, bias)
            losses.append(F.cross_entropy(logits, target[lo:lo + self.chunk], ignore_index=-100, reduction="none"))
        return torch.cat(losses)

    def __call__(self, lm: torch.nn.Module, *args: Any, **kwargs: Any):
        kw = self._kwargs(args, kwargs)
        labels = kw.pop("labels", None)
        keep = kw.pop("logits_to_keep", 0)
        if not self.inner_takes_any:
            kw = {k: v for k, v in kw.items() if k in self.inner_names}
        hidden = lm.model(**kw)[0]
        sel = slice(-keep, None) if isinstance(keep, int) else keep
        hidden = hidden[:, sel, :] if hidden.dim() == 3 else hidden[sel, :]
        if labels is None:
            result = {"loss": None, "logits": lm.lm_head(hidden)}
        else:
            result = {"loss": self._token_losses(lm, hidden, labels, keep), "logits": None}
        if self.output_cls is None:
            return result
        return self.output_cls(**{k: v for k, v in result.items() if k in self.output_fields})


def apply_chunked_token_loss_patch(model: torch.nn.Module, *, chunk_size: int = 4096,
                                   output_cls: Optional[type] = None) -> torch.nn.Module:
    """Make a causal LM return the unreduced per-token loss without materialising full logits.

    This engine's own models already compute the loss with the fused linear + cross-entropy
    kernels; for them only the chunk size is set.  Any other model exposing ``.model`` and
    ``.lm_head`` gets :class:`_ChunkedLossForward` as its ``forward``."""
    if chunk_size <= 0:
        raise ValueError("chunk_size must be positive.")
    if hasattr(model, "loss_chunk_size"):
        model.loss_chunk_size = int(chunk_size)
        return model
    if not (hasattr(model, "model") and hasattr(model, "lm_head")):
        raise ValueError("Chunked token loss patch requires the model to expose `.model` and `.lm_head`.")
    impl = _ChunkedLossForward(model, chunk_size, output_cls)

    def forward(self, *args: Any, **kwargs: Any):
        return impl(self, *args, **kwargs)

    forward.__signature__ = impl.outer_sig
    model.forward = MethodType(forward, model)
    return model
