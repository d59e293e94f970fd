"""Multimodal data pipeline pieces."""

from .collator import MLLMBatchCollator
from .data import MLLMDataKit
from .guard import MLLMModelInputGuard, MLLMRawRowGuard, MLLMSampleGuard, MLLMTextOnlyBatchGuard
from .media import MLLMMediaHandler, MLLMMediaTypeHandler, RenderedMedia, empty_model_sample
from .packing import MLLMPackingAssembler, build_packed_block_causal_mask
from .qwen import (QwenImageHandler, QwenVLChatSchemaHandler, QwenVLImageProcessor, QwenVLMediaHandler,
                   QwenVLProcessor, QwenVLTokenizationHandler, smart_resize)
from .sample import MLLMPack, MLLMSample
from .schema import MLLMSchemaHandler, SyntheticVLSchemaHandler
from .spec import (MLLMDataSpec, MLLMDistributionSpec, MLLMLoaderSpec, MLLMPackingSpec, MLLMSampleSpec,
                   MLLMSourceSpec)
from .tokenization import MLLMTokenizationHandler
from .types import MLLMMediaSlot, MLLMSegment, ModelInputs
