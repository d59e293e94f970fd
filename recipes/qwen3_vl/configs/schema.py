"""Qwen3-VL recipe config (reference: recipes/qwen3_vl/configs/schema.py:10-212).

Same fields and validation as the reference; additions: ``data.dataset_source``
(``lance`` / ``json`` / ``parquet`` / ``synthetic_mm``), ``model.load_pretrained_model``,
``model.gradient_checkpointing.num_layers`` and ``model.config_overrides``.
"""

from __future__ import annotations

from typing import Any, Literal, Optional

from pydantic import BaseModel, ConfigDict, Field, field_validator

from mvp_engine.config.schema import BaseEngineConfig, BaseLoopConfig, BaseOptimConfig

from recipes.qwen3.configs.schema import resolve_batching


class Qwen3VLDataConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    train_path: str = "./data/mvp-engine-vlm-dev-data/meta.json"
    dataset_source: str = "lance"
    ref_columns: list[str] = Field(default_factory=lambda: ["images"])
    thinking_mode: bool | None | Literal["non-empty"] = "non-empty"
    packing_selection_strategy: Literal["random", "best_fit"] = "best_fit"
    packing_open_pack_limit: int = Field(8, ge=1)
    packing_buffer_size: int = Field(64, ge=0)
    max_seq_len: int = Field(2048, ge=1)
    batch_size: int = 1
    num_workers: int = Field(0, ge=0)

    @field_validator("train_path", mode="before")
    @classmethod
    def _path(cls, v: Any) -> Any:
        if not isinstance(v, str):
            raise TypeError("`data.train_path` must be a string.")
        if not v.strip():
            raise ValueError("`data.train_path` must not be empty.")
        return v.strip()

    @field_validator("batch_size")
    @classmethod
    def _bs(cls, v: int) -> int:
        if v == 0 or v < -1:
            raise ValueError("`data.batch_size` must be positive or exactly -1.")
        return v

    @field_validator("thinking_mode", mode="before")
    @classmethod
    def _thinking(cls, v: Any) -> Any:
        if v is None or isinstance(v, bool):
            return v
        if isinstance(v, str) and v.strip().lower() in {"non-empty", "non_empty", "nonempty"}:
            return "non-empty"
        if isinstance(v, str) and v.strip().lower() in {"true", "false"}:
            return v.strip().lower() == "true"
        raise ValueError("`data.thinking_mode` must be a bool, null, or 'non-empty'.")


class Qwen3VLGradientCheckpointingConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    enabled: bool = False
    use_reentrant: bool = False
    num_layers: Optional[int] = None


class Qwen3VLCompileConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    enabled: bool = False
    backend: str = "inductor"
    mode: str = "default"


class Qwen3VLModelConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    pretrained_model_name_or_path: str = "Qwen/Qwen3-VL-8B-Instruct"
    attn_implementation: Literal["eager", "sdpa", "flash_attention_2", "mvp_flash_varlen"] = "flash_attention_2"
    load_pretrained_model: bool = False
    image_max_pixels: Optional[int] = Field(None, ge=1)
    gradient_checkpointing: Qwen3VLGradientCheckpointingConfig = Field(
        default_factory=Qwen3VLGradientCheckpointingConfig)
    freeze_vit: bool = False
    freeze_projector: bool = False
    freeze_llm: bool = False
    compile: Qwen3VLCompileConfig = Field(default_factory=Qwen3VLCompileConfig)
    config_overrides: dict[str, Any] = Field(default_factory=dict)

    @field_validator("pretrained_model_name_or_path", mode="before")
    @classmethod
    def _name(cls, v: Any) -> Any:
        if not isinstance(v, str):
            raise TypeError("`model.pretrained_model_name_or_path` must be a string.")
        if not v.strip():
            raise ValueError("`model.pretrained_model_name_or_path` must not be empty.")
        return v.strip()


class Qwen3VLOptimConfig(BaseOptimConfig):
    model_config = ConfigDict(frozen=False)

    optimizer: str = "AdamW"
    gradient_accumulation_steps: int = 1  # type: ignore[assignment]
    global_batch_size: Optional[int] = Field(None, ge=1)
    loss_spike_skip_multiplier: Optional[float] = Field(None, gt=0.0)
    loss_spike_skip_window_size: int = Field(8, ge=1)
    loss_spike_skip_min_history: int = Field(3, ge=1)

    @field_validator("gradient_accumulation_steps")
    @classmethod
    def _ga(cls, v: int) -> int:
        if v == 0 or v < -1:
            raise ValueError("`optim.gradient_accumulation_steps` must be positive or exactly -1.")
        return v


class Qwen3VLLoopConfig(BaseLoopConfig):
    model_config = ConfigDict(frozen=False)

    total_steps: int = -1  # type: ignore[assignment]

    @field_validator("total_steps")
    @classmethod
    def _steps(cls, v: int) -> int:
        if v == 0 or v < -1:
            raise ValueError("`loop.total_steps` must be positive or exactly -1.")
        return v


class Qwen3VLConfig(BaseEngineConfig):
    model_config = ConfigDict(frozen=False, extra="allow")

    data: Qwen3VLDataConfig = Field(default_factory=Qwen3VLDataConfig)
    model: Qwen3VLModelConfig = Field(default_factory=Qwen3VLModelConfig)
    optim: Qwen3VLOptimConfig = Field(default_factory=Qwen3VLOptimConfig)
    loop: Qwen3VLLoopConfig = Field(default_factory=Qwen3VLLoopConfig)

    def resolve_batching_config(self, *, data_parallel_world_size: int) -> None:
        resolve_batching(self, data_parallel_world_size)
