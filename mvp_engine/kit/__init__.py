"""Reusable training kits, resolved lazily (reference: mvp_engine/kit/__init__.py:72-149)."""

from importlib import import_module

_EXPORTS = {
    **{n: ".llm" for n in (
        "LLMBatchCollator", "LLMDataKit", "LLMDataSpec", "LLMDistributionSpec", "LLMLoaderSpec", "LLMModelKit",
        "LLMPack", "LLMPackingAssembler", "LLMPackingSpec", "LLMPretrainTextSchemaHandler",
        "LLMPretrainTextTokenizationHandler", "LLMSample", "LLMSampleSpec", "LLMSchemaHandler", "LLMSegment",
        "LLMSourceSpec", "LLMStepEstimateResult", "LLMStepEstimationKit", "LLMTokenizationHandler",
        "LLMTokenIdsSchemaHandler", "QwenChatSchemaHandler", "QwenChatTokenizationHandler")},
    **{n: ".mllm" for n in (
        "Confidence", "MLLMBatchCollator", "MLLMDataKit", "MLLMDataSpec", "MLLMDistributionSpec", "MLLMLoaderSpec",
        "MLLMMediaHandler", "MLLMMediaSlot", "MLLMMediaTypeHandler", "MLLMModelKit", "MLLMPack",
        "MLLMPackingAssembler", "MLLMPackingSpec", "MLLMSample", "MLLMSampleSpec", "MLLMSchemaHandler",
        "MLLMSegment", "MLLMSourceSpec", "MLLMStepEstimationKit", "MLLMTextOnlyBatchGuard",
        "MLLMTokenizationHandler", "ModelInputs", "QwenImageHandler", "QwenVLChatSchemaHandler",
        "QwenVLMediaHandler", "QwenVLTokenizationHandler", "StepEstimateResult")},
    "LossGuard": ".loss.loss",
    "LossKit": ".loss.loss",
    "PerTokenLossGuard": ".loss.token_loss",
    "TokenLossStats": ".loss.token_loss",
    "TokenNormedLossKit": ".loss.token_loss",
    "apply_chunked_token_loss_patch": ".loss.token_loss",
    "MFUKit": ".perf.mfu",
    "LigerKernelKit": ".model",
    "LigerKernelReport": ".model",
    "LigerPatch": ".model",
    "OptimKit": ".optim",
    "StepCountResult": ".util",
    "StepCountingKit": ".util",
}

__all__ = list(_EXPORTS)


def __getattr__(name: str):
    if name not in _EXPORTS:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(import_module(_EXPORTS[name], __name__), name)
    globals()[name] = value
    return value
