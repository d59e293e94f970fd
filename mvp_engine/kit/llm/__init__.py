"""Text-LM kits."""

from .data import *  # noqa: F401,F403
from .data import (LLMBatchCollator, LLMDataKit, LLMDataSpec, LLMDistributionSpec, LLMLoaderSpec, LLMPack,
                   LLMPackingAssembler, LLMPackingSpec, LLMPretrainTextSchemaHandler,
                   LLMPretrainTextTokenizationHandler, LLMSample, LLMSampleSpec, LLMSchemaHandler, LLMSegment,
                   LLMSourceSpec, LLMTokenIdsSchemaHandler, LLMTokenizationHandler, ModelInputs,
                   QwenChatSchemaHandler, QwenChatTokenizationHandler)
from .model import LLMModelKit
from .utils import LLMStepEstimateResult, LLMStepEstimationKit
