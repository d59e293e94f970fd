from .step_counting import StepCountingKit, StepCountResult, samples_per_step

__all__ = ["StepCountingKit", "StepCountResult", "samples_per_step"]
