"""Gradient accumulation, loss scaling and global-norm clipping
(reference: mvp_engine/utils/training.py:116-349).

``accumulate_gradients`` understands three wrappers: torch DDP (``no_sync``),
torch FSDP2 (``set_requires_gradient_sync``) and the engine's native
flat-buffer data-parallel wrapper (``set_requires_gradient_sync`` as well).
``clip_grad_norm_`` computes the global norm over local shards: DTensor
gradients are grouped by mesh/placement and reduced over every sharded or
partial mesh dimension; the native wrapper computes its norm over its flat
fp32 gradient shards with one all-reduce.
"""

from __future__ import annotations

import math
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Generator, Iterable, Union

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.nn.parallel import DistributedDataParallel as DDP

try:
    from torch.distributed.fsdp import FSDPModule
except Exception:  # pragma: no cover
    FSDPModule = ()  # type: ignore[assignment]

try:
    from torch.distributed.tensor import DTensor
except Exception:  # pragma: no cover
    DTensor = ()  # type: ignore[assignment]


@dataclass
class GradientAccumulationState:
    """Counts micro-batches; ``advance`` returns True on the micro-batch that syncs."""

    gradient_accumulation_steps: int
    micro_step: int = 0

    def advance(self, skip_increase: bool = False) -> bool:
        if not skip_increase:
            self.micro_step += 1
        if self.micro_step % max(1, self.gradient_accumulation_steps) == 0:
            self.micro_step = 0
            return True
        return False


@contextmanager
def accumulate_gradients(model: Union[nn.Module, DDP], sync: bool) -> Generator[None, None, None]:
    base = getattr(model, "_orig_mod", model)
    if isinstance(base, DDP):
        if sync:
            yield
        else:
            with base.no_sync():
                yield
        return
    setter = getattr(base, "set_requires_gradient_sync", None)
    if callable(setter):
        setter(sync)
    yield


class GradientScaler:
    """Loss scaling only for fp16 on CUDA; a pass-through for bf16/fp32."""

    def __init__(self, enabled: bool = True, dtype: torch.dtype = torch.float16, device: str = "cuda",
                 init_scale: float = 65536.0, growth_factor: float = 2.0, backoff_factor: float = 0.5,
                 growth_interval: int = 2000) -> None:
        self._enabled = enabled
        self._dtype = dtype
        self._device = device
        use = enabled and dtype == torch.float16 and device == "cuda" and torch.cuda.is_available()
        self._scaler = (torch.amp.GradScaler(device=device, init_scale=init_scale, growth_factor=growth_factor,
                                             backoff_factor=backoff_factor, growth_interval=growth_interval)
                        if use else None)

    def scale(self, loss: torch.Tensor) -> torch.Tensor:
        return self._scaler.scale(loss) if self._scaler is not None else loss

    def unscale_(self, optimizer) -> None:
        if self._scaler is not None:
            self._scaler.unscale_(optimizer)

    def step(self, optimizer) -> None:
        if self._scaler is not None:
            self._scaler.step(optimizer)
        else:
            optimizer.step()

    def update(self) -> None:
        if self._scaler is not None:
            self._scaler.update()

    def get_scale(self) -> float:
        return float(self._scaler.get_scale()) if self._scaler is not None else 1.0

    def state_dict(self) -> dict:
        return self._scaler.state_dict() if self._scaler is not None else {}

    def load_state_dict(self, state_dict: dict) -> None:
        if self._scaler is not None and state_dict:
            self._scaler.load_state_dict(state_dict)


def _local(t: torch.Tensor) -> torch.Tensor:
    if isinstance(t, DTensor):
        loc = t.to_local()
        wait = getattr(loc, "wait", None)
        return wait() if callable(wait) else loc
    return t


def _mesh_key(g: torch.Tensor) -> tuple:
    if not isinstance(g, DTensor):
        return ("local",)
    m = g.device_mesh
    return ("dtensor", m.device_type, tuple(m.mesh.shape), tuple(m.mesh.reshape(-1).tolist()),
            tuple(m.mesh_dim_names or ()), tuple(repr(p) for p in g.placements))


def _group_norm(grads: list[torch.Tensor], p: float) -> torch.Tensor:
    locs = [_local(g).detach() for g in grads]
    if math.isinf(p):
        val = torch.stack([torch.linalg.vector_norm(x, ord=p, dtype=torch.float32) for x in locs]).amax()
        op = dist.ReduceOp.MAX
    else:
        val = torch.stack([torch.linalg.vector_norm(x, ord=p, dtype=torch.float32) ** p for x in locs]).sum()
        op = dist.ReduceOp.SUM
    g0 = grads[0]
    if isinstance(g0, DTensor):
        dev = torch.device("cuda", torch.cuda.current_device()) if g0.device_mesh.device_type == "cuda" \
            else torch.device(g0.device_mesh.device_type)
        val = val.to(dev)
        for dim, placement in enumerate(g0.placements):
            if placement.is_shard() or placement.is_partial():
                dist.all_reduce(val, op=op, group=g0.device_mesh.get_group(dim))
    if not math.isinf(p):
        val = val ** (1.0 / p)
    return val.to(device=locs[0].device, dtype=torch.float32)


@torch.no_grad()
def clip_grad_norm_(parameters: Union[nn.Module, Iterable[torch.Tensor], torch.Tensor], max_norm: float,
                    norm_type: float = 2.0) -> torch.Tensor:
    """Scale gradients in place so their global ``norm_type`` norm is at most ``max_norm``.

    Returns the total norm before clipping.
    """
    if isinstance(parameters, nn.Module):
        native = getattr(parameters, "clip_grad_norm_", None)
        if callable(native):
            return native(max_norm, norm_type)
        parameters = parameters.parameters()
    params = [parameters] if isinstance(parameters, torch.Tensor) else list(parameters)
    params = [p for p in params if p.grad is not None]
    if not params:
        return torch.tensor(0.0)
    groups: dict[tuple, list[torch.Tensor]] = {}
    for p in params:
        groups.setdefault(_mesh_key(p.grad), []).append(p)
    norms = []
    for ps in groups.values():
        grads = [p.grad for p in ps]
        if isinstance(grads[0], DTensor):
            norms.append(_group_norm(grads, norm_type))
        else:
            norms.append(torch.nn.utils.get_total_norm(grads, norm_type).float())
    dev = norms[0].device
    stacked = torch.stack([n.to(dev) for n in norms])
    total = stacked.amax() if math.isinf(norm_type) else torch.linalg.vector_norm(stacked, ord=norm_type)
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    for ps in groups.values():
        for p in ps:
            loc = _local(p.grad)
            loc.mul_(coef.to(device=loc.device, dtype=loc.dtype))
    return total
