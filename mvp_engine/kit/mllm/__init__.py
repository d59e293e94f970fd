"""Multimodal kits."""

from .data import *  # noqa: F401,F403
from .data import (MLLMBatchCollator, MLLMDataKit, MLLMDataSpec, MLLMDistributionSpec, MLLMLoaderSpec,
                   MLLMMediaHandler, MLLMMediaSlot, MLLMMediaTypeHandler, MLLMPack, MLLMPackingAssembler,
                   MLLMPackingSpec, MLLMSample, MLLMSampleSpec, MLLMSchemaHandler, MLLMSegment, MLLMSourceSpec,
                   MLLMTextOnlyBatchGuard, MLLMTokenizationHandler, ModelInputs, QwenImageHandler,
                   QwenVLChatSchemaHandler, QwenVLTokenizationHandler)
from .data.qwen import QwenVLMediaHandler
from .model import MLLMModelKit
from .utils import Confidence, MLLMStepEstimationKit, StepEstimateResult
