"""OpenBee config (reference: recipes/openbee/configs/schema.py): the Qwen3-VL recipe schema with an
empty default ``data.train_path`` (each stage names its own data)."""

from __future__ import annotations

from pydantic import Field

from recipes.qwen3_vl.configs.schema import (Qwen3VLCompileConfig, Qwen3VLConfig, Qwen3VLDataConfig,
                                             Qwen3VLGradientCheckpointingConfig, Qwen3VLLoopConfig,
                                             Qwen3VLModelConfig, Qwen3VLOptimConfig)

# The reference spells out every section for OpenBee; here the sections are the Qwen3-VL ones under the
# reference's class names, so code that imports them by name keeps working.
OpenBeeGradientCheckpointingConfig = Qwen3VLGradientCheckpointingConfig
OpenBeeCompileConfig = Qwen3VLCompileConfig
OpenBeeModelConfig = Qwen3VLModelConfig
OpenBeeOptimConfig = Qwen3VLOptimConfig
OpenBeeLoopConfig = Qwen3VLLoopConfig


class OpenBeeDataConfig(Qwen3VLDataConfig):
    train_path: str = "synthetic://mm"


class OpenBeeConfig(Qwen3VLConfig):
    data: OpenBeeDataConfig = Field(default_factory=OpenBeeDataConfig)
