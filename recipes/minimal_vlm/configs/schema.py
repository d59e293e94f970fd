"""Minimal VLM config (reference: recipes/minimal_vlm/configs/schema.py:10-53); adds
``data.dataset_source`` (``parquet`` or ``synthetic_mm``) and ``model.config_overrides``."""

from __future__ import annotations

from typing import Any, Optional

from pydantic import BaseModel, ConfigDict, Field, field_validator

from mvp_engine.config.schema import BaseEngineConfig


class MinimalVLMDataConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    train_path: Optional[str] = "./data/minimal_vlm/demo.parquet"
    dataset_source: str = "parquet"
    max_seq_len: int = Field(2048, ge=1)
    batch_size: int = Field(1, ge=1)
    num_workers: int = Field(0, ge=0)

    @field_validator("train_path", mode="before")
    @classmethod
    def _path(cls, v: Any) -> Any:
        if v is None:
            return v
        if not isinstance(v, str) or not v.strip():
            raise ValueError("`data.train_path` must be a non-empty string or null.")
        return v.strip()


class MinimalVLMModelConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    pretrained_model_name_or_path: str = "Qwen/Qwen3-VL-2B-Instruct"
    load_pretrained_model: bool = False
    image_max_pixels: Optional[int] = None
    config_overrides: dict[str, Any] = Field(default_factory=dict)

    @field_validator("pretrained_model_name_or_path", mode="before")
    @classmethod
    def _name(cls, v: Any) -> Any:
        if not isinstance(v, str) or not v.strip():
            raise ValueError("`model.pretrained_model_name_or_path` must be a non-empty string.")
        return v.strip()


class MinimalVLMConfig(BaseEngineConfig):
    model_config = ConfigDict(frozen=False, extra="allow")

    data: MinimalVLMDataConfig = Field(default_factory=MinimalVLMDataConfig)
    model: MinimalVLMModelConfig = Field(default_factory=MinimalVLMModelConfig)
