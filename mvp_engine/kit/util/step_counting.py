"""Exact optimizer-step counting over a finite dataset (reference: mvp_engine/kit/util/step_counting.py:22-142)."""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from ...utils.log import simple_info

SampleCounter = Callable[[object], int]


def samples_per_step(batch_size: int, gradient_accumulation_steps: int) -> int:
    if batch_size <= 0 or gradient_accumulation_steps <= 0:
        raise ValueError("batch_size and gradient_accumulation_steps must be positive.")
    return int(batch_size) * int(gradient_accumulation_steps)


def resolve_reduce_device(*, dp_world_size: int, dp_group=None, device: Optional[torch.device] = None) -> torch.device:
    if device is not None:
        return torch.device(device)
    if dist.is_available() and dist.is_initialized() and dist.get_backend(dp_group) == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


@dataclass(frozen=True, slots=True)
class StepCountResult:
    total_steps: int
    total_samples: int
    samples_per_step: int


class _Counter:
    def __init__(self, fn: SampleCounter) -> None:
        self.fn = fn
        self.total = 0

    def push(self, item: object) -> bool:
        n = int(self.fn(item))
        if n <= 0:
            raise RuntimeError("Sample counter must return a positive integer.")
        self.total += n
        return True

    def finish(self) -> int:
        return self.total


def reduce_counts(local: int, *, per_step: int, dp_world_size: int, dp_group=None,
                  device: Optional[torch.device] = None) -> tuple[int, int, bool]:
    """Global (samples SUM, steps MAX, all-ranks-nonempty MIN)."""
    steps = math.ceil(local / per_step)
    if dp_world_size <= 1 or not (dist.is_available() and dist.is_initialized()):
        return local, steps, local > 0
    dev = resolve_reduce_device(dp_world_size=dp_world_size, dp_group=dp_group, device=device)
    t = torch.tensor([local, steps, int(local > 0)], dtype=torch.long, device=dev)
    s, m, n = t[0:1].clone(), t[1:2].clone(), t[2:3].clone()
    dist.all_reduce(s, op=dist.ReduceOp.SUM, group=dp_group)
    dist.all_reduce(m, op=dist.ReduceOp.MAX, group=dp_group)
    dist.all_reduce(n, op=dist.ReduceOp.MIN, group=dp_group)
    return int(s.item()), int(m.item()), bool(n.item())


class StepCountingKit:
    def __init__(self, *, sample_counter: SampleCounter = lambda _item: 1) -> None:
        self.sample_counter = sample_counter

    def count_total_steps(self, dataset: object, *, batch_size: int, gradient_accumulation_steps: int,
                          data_parallel_world_size: int, data_parallel_group=None,
                          device: Optional[torch.device] = None) -> StepCountResult:
        per = samples_per_step(batch_size, gradient_accumulation_steps)
        consume = getattr(dataset, "consume", None)
        if not callable(consume):
            raise TypeError("StepCountingKit requires a dataset with a consume(factory) method.")
        local = int(consume(lambda _ctx: _Counter(self.sample_counter)))
        total, steps, nonempty = reduce_counts(local, per_step=per, dp_world_size=data_parallel_world_size,
                                               dp_group=data_parallel_group, device=device)
        if total <= 0:
            raise RuntimeError("Step counting found no training samples.")
        if not nonempty:
            raise RuntimeError("Step counting found a data-parallel rank with no training samples.")
        simple_info(f"Step counting: total_samples={total}, samples_per_step={per}, "
                    f"dp_world_size={data_parallel_world_size}, total_steps={steps}")
        return StepCountResult(steps, total, per)
