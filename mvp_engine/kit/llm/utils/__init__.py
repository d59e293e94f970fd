from .step_estimation import LLMStepEstimateResult, LLMStepEstimationKit

__all__ = ["LLMStepEstimateResult", "LLMStepEstimationKit"]
