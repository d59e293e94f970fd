from .step_estimation import Confidence, MLLMStepEstimationKit, StepEstimateResult

__all__ = ["Confidence", "MLLMStepEstimationKit", "StepEstimateResult"]
