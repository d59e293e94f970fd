"""Exact optimizer-step count of a finite packed text dataset.

Public API of the reference's ``mvp_engine/kit/llm/utils/step_estimation.py:24-56``.  The count
comes from one pass over the (packed) dataset through :class:`StepCountingKit`, which reduces
the per-rank pack counts over the data-parallel group; this kit only reshapes and reports it.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

from ....utils.log import simple_info
from ...util.step_counting import StepCountingKit


@dataclass(frozen=True)
class LLMStepEstimateResult:
    total_steps: int
    total_packed_samples: int
    samples_per_step: int
    exact: bool = True


class LLMStepEstimationKit:
    def __init__(self, counter: Optional[StepCountingKit] = None) -> None:
        self.counter = counter or StepCountingKit()

    def estimate_total_steps(self, dataset: object, *, batch_size: int, gradient_accumulation_steps: int,
                             data_parallel_world_size: int, data_parallel_group=None,
                             device=None) -> LLMStepEstimateResult:
        count = self.counter.count_total_steps(dataset, batch_size=batch_size,
                                               gradient_accumulation_steps=gradient_accumulation_steps,
                                               data_parallel_world_size=data_parallel_world_size,
                                               data_parallel_group=data_parallel_group, device=device)
        result = LLMStepEstimateResult(total_steps=count.total_steps, total_packed_samples=count.total_samples,
                                       samples_per_step=count.samples_per_step)
        facts = {"exact": result.exact, "packed_samples": result.total_packed_samples,
                 "samples_per_step": result.samples_per_step, "dp_world_size": data_parallel_world_size,
                 "total_steps": result.total_steps}
        simple_info("LLM step estimation: " + ", ".join(f"{k}={v}" for k, v in facts.items()))
        return result
