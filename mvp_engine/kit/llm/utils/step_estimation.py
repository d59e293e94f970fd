"""Exact step count of a finite packed text dataset (reference: mvp_engine/kit/llm/utils/step_estimation.py:24-56)."""

from __future__ import annotations

from dataclasses import dataclass

from ...util.step_counting import StepCountingKit, samples_per_step
from ....utils.log import simple_info


@dataclass(frozen=True, slots=True)
class LLMStepEstimateResult:
    total_steps: int
    total_packed_samples: int
    samples_per_step: int
    exact: bool = True


class LLMStepEstimationKit:
    def estimate_total_steps(self, dataset: object, *, batch_size: int, gradient_accumulation_steps: int,
                             data_parallel_world_size: int, data_parallel_group=None, device=None) -> LLMStepEstimateResult:
        per = samples_per_step(batch_size, gradient_accumulation_steps)
        r = StepCountingKit().count_total_steps(dataset, batch_size=batch_size,
                                                gradient_accumulation_steps=gradient_accumulation_steps,
                                                data_parallel_world_size=data_parallel_world_size,
                                                data_parallel_group=data_parallel_group, device=device)
        simple_info(f"LLM step estimation: exact=True, packed_samples={r.total_samples}, samples_per_step={per}, "
                    f"dp_world_size={data_parallel_world_size}, total_steps={r.total_steps}")
        return LLMStepEstimateResult(r.total_steps, r.total_samples, per)
