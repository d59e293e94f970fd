"""Text-LM data pipeline pieces."""

from .collator import LLMBatchCollator, varlen_metadata
from .data import IGNORE_INDEX, LLMDataKit
from .guard import CheckResult, LLMModelInputGuard, LLMRawRowGuard, LLMSampleGuard
from .packing import LLMPackingAssembler, build_packed_block_causal_mask
from .qwen import QwenChatSchemaHandler, QwenChatTokenizationHandler
from .sample import LLMPack, LLMSample, LLMSampleAssembler
from .schema import LLMPretrainTextSchemaHandler, LLMSchemaHandler, LLMTokenIdsSchemaHandler
from .spec import (LLMDataSpec, LLMDistributionSpec, LLMLoaderSpec, LLMPackingSpec, LLMSampleSpec,
                   LLMSourceSpec)
from .tokenization import LLMPretrainTextTokenizationHandler, LLMTokenizationHandler
from .types import LLMSegment, ModelInputs
