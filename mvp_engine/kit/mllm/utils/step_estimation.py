"""Optimizer-step estimation for packed multimodal data (reference: mvp_engine/kit/mllm/utils/step_estimation.py:30-332).

Packing merges several source rows into one packed sample, so the number of
steps of an epoch is estimated from the packed/source compression ratio: the
local stream is consumed until a window of recent ratio estimates is stable
enough for the target ``Confidence`` (relative spread below 5% / 1% / 0.1%),
or until the rank's share of source rows is exhausted (exact).  Ranks vote
every ``sync_interval`` packs (all-reduce MIN) so all stop together; the
result is reduced across ranks (packs SUM, steps MAX).
"""

from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass
from enum import IntEnum
from typing import Optional

import torch
import torch.distributed as dist

from ...util.step_counting import resolve_reduce_device, samples_per_step
from ....utils.log import simple_info


class Confidence(IntEnum):
    LOW = 0
    MEDIUM = 1
    HIGH = 2
    VERY_HIGH = 3


_SPREAD = ((0.001, Confidence.VERY_HIGH), (0.01, Confidence.HIGH), (0.05, Confidence.MEDIUM))


@dataclass(frozen=True, slots=True)
class StepEstimateResult:
    total_steps: int
    estimated_total_packed_samples: float
    seen_packed_samples: int
    seen_source_samples: int
    total_source_samples: int
    compression_ratio: float
    confidence: Confidence
    exact: bool


def _confidence(estimates) -> Confidence:
    if len(estimates) < 2:
        return Confidence.LOW
    mean = sum(estimates) / len(estimates)
    if mean <= 0:
        return Confidence.LOW
    spread = (max(estimates) - min(estimates)) / mean
    for limit, conf in _SPREAD:
        if spread <= limit:
            return conf
    return Confidence.LOW


class MLLMStepEstimationKit:
    def count_source_samples(self, item: object) -> int:
        n = item.get("source_sample_num", 1) if isinstance(item, dict) else getattr(item, "source_sample_num", 1)
        return int(n.sum()) if isinstance(n, torch.Tensor) else int(n)

    def estimate_total_steps(self, dataset: object, *, total_source_samples: int, batch_size: int,
                             gradient_accumulation_steps: int, data_parallel_world_size: int,
                             data_parallel_group=None, device: Optional[torch.device] = None,
                             target_confidence: Confidence = Confidence.HIGH, confidence_window_size: int = 100,
                             sync_interval: int = 100) -> StepEstimateResult:
        if total_source_samples <= 0:
            raise ValueError("`total_source_samples` must be a positive dataset-wide source-row count.")
        if confidence_window_size <= 0 or sync_interval <= 0:
            raise ValueError("window and sync interval must be positive")
        per = samples_per_step(batch_size, gradient_accumulation_steps)
        target = math.ceil(total_source_samples / data_parallel_world_size)
        distributed = data_parallel_world_size > 1 and dist.is_available() and dist.is_initialized()
        dev = resolve_reduce_device(dp_world_size=data_parallel_world_size, dp_group=data_parallel_group,
                                    device=device)
        packs = srcs = 0
        window: deque = deque(maxlen=confidence_window_size)
        conf = Confidence.LOW
        exact = True
        for item in dataset:
            packs += 1
            srcs += self.count_source_samples(item)
            if srcs > 0:
                window.append(packs * target / srcs)
            conf = _confidence(window)
            local_done = conf >= target_confidence or srcs >= target
            if packs % sync_interval == 0 or local_done:
                if distributed:
                    vote = torch.tensor([int(local_done)], device=dev)
                    dist.all_reduce(vote, op=dist.ReduceOp.MIN, group=data_parallel_group)
                    local_done = bool(vote.item())
                if local_done:
                    exact = srcs >= target and conf < target_confidence
                    break
        est_packs = packs * target / max(1, srcs) if not exact else float(packs)
        steps = math.ceil(est_packs / per)
        vals = torch.tensor([est_packs, float(packs), float(srcs)], dtype=torch.float64, device=dev)
        st = torch.tensor([steps, int(packs > 0)], dtype=torch.long, device=dev)
        if distributed:
            dist.all_reduce(vals, group=data_parallel_group)
            mx = st[0:1].clone()
            mn = st[1:2].clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=data_parallel_group)
            dist.all_reduce(mn, op=dist.ReduceOp.MIN, group=data_parallel_group)
            st = torch.cat([mx, mn])
        res = StepEstimateResult(total_steps=int(st[0]), estimated_total_packed_samples=float(vals[0]),
                                 seen_packed_samples=int(vals[1]), seen_source_samples=int(vals[2]),
                                 total_source_samples=int(total_source_samples),
                                 compression_ratio=float(vals[1]) / max(1.0, float(vals[2])), confidence=conf,
                                 exact=exact)
        if res.seen_packed_samples <= 0:
            raise RuntimeError("MLLM step estimation found no packed training samples.")
        if not bool(st[1]):
            raise RuntimeError("MLLM step estimation found a data-parallel rank with no packed samples.")
        simple_info(f"MLLM step estimation: exact={res.exact}, confidence={res.confidence.name}, "
                    f"seen_packed={res.seen_packed_samples}, total_steps={res.total_steps}")
        return res
