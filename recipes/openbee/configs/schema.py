"""OpenBee config (reference: recipes/openbee/configs/schema.py): the Qwen3-VL recipe schema with an
empty default ``data.train_path`` (each stage names its own data)."""

from __future__ import annotations

from pydantic import Field

from recipes.qwen3_vl.configs.schema import Qwen3VLConfig, Qwen3VLDataConfig


class OpenBeeDataConfig(Qwen3VLDataConfig):
    train_path: str = "synthetic://mm"


class OpenBeeConfig(Qwen3VLConfig):
    data: OpenBeeDataConfig = Field(default_factory=OpenBeeDataConfig)
