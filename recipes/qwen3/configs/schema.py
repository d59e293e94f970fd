"""Qwen3 recipe config (reference: recipes/qwen3/configs/schema.py:1-182).

Same fields and batching rules as the reference; additions: ``data.dataset_source``
(e.g. ``synthetic_text``), ``model.gradient_checkpointing.num_layers`` (recompute
only the first N layers) and ``model.config_overrides`` (architecture fields
on top of the preset / config.json).
"""

from __future__ import annotations

from typing import Any, Literal, Optional

from pydantic import BaseModel, ConfigDict, Field, field_validator

from mvp_engine.config.schema import BaseEngineConfig, BaseLoopConfig, BaseOptimConfig


class Qwen3DataConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    train_path: str = "synthetic://text"
    dataset_source: str = "lance"
    text_field: str = "data"
    packing_tail_policy: Literal["drop", "pad"] = "drop"
    packing_isolate_attention: bool = False
    packing_isolate_position_ids: bool = False
    max_seq_len: int = Field(8192, ge=1)
    batch_size: int = 1
    num_workers: int = Field(0, ge=0)

    @field_validator("train_path", mode="before")
    @classmethod
    def _path(cls, v: Any) -> Any:
        if v is None:
            return v
        if not isinstance(v, str):
            raise TypeError("`data.train_path` must be a string or null.")
        if not v.strip():
            raise ValueError("`data.train_path` must not be empty.")
        return v.strip()

    @field_validator("batch_size")
    @classmethod
    def _bs(cls, v: int) -> int:
        if v == 0 or v < -1:
            raise ValueError("`data.batch_size` must be positive or exactly -1.")
        return v


class Qwen3GradientCheckpointingConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    enabled: bool = False
    use_reentrant: bool = False
    num_layers: Optional[int] = None


class Qwen3CompileConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    enabled: bool = False
    backend: str = "inductor"
    mode: str = "default"


class Qwen3ModelConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    pretrained_model_name_or_path: str = "Qwen/Qwen3-8B-Base"
    attn_implementation: Literal["eager", "sdpa", "flash_attention_2", "mvp_flash_varlen"] = "flash_attention_2"
    load_pretrained_model: bool = False
    gradient_checkpointing: Qwen3GradientCheckpointingConfig = Field(default_factory=Qwen3GradientCheckpointingConfig)
    freeze_llm: bool = False
    compile: Qwen3CompileConfig = Field(default_factory=Qwen3CompileConfig)
    config_overrides: dict[str, Any] = Field(default_factory=dict)

    @field_validator("pretrained_model_name_or_path", mode="before")
    @classmethod
    def _name(cls, v: Any) -> Any:
        if not isinstance(v, str):
            raise TypeError("`model.pretrained_model_name_or_path` must be a string.")
        if not v.strip():
            raise ValueError("`model.pretrained_model_name_or_path` must not be empty.")
        return v.strip()


class Qwen3OptimConfig(BaseOptimConfig):
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


class Qwen3LoopConfig(BaseLoopConfig):
    model_config = ConfigDict(frozen=False)

    total_steps: int = 10000  # type: ignore[assignment]

    @field_validator("total_steps")
    @classmethod
    def _steps(cls, v: int) -> int:
        if v == 0 or v < -1:
            raise ValueError("`loop.total_steps` must be positive or exactly -1.")
        return v


class Qwen3Config(BaseEngineConfig):
    model_config = ConfigDict(frozen=False, extra="allow")

    data: Qwen3DataConfig = Field(default_factory=Qwen3DataConfig)
    model: Qwen3ModelConfig = Field(default_factory=Qwen3ModelConfig)
    optim: Qwen3OptimConfig = Field(default_factory=Qwen3OptimConfig)
    loop: Qwen3LoopConfig = Field(default_factory=Qwen3LoopConfig)

    def resolve_batching_config(self, *, data_parallel_world_size: int) -> None:
        """Infer ``data.batch_size`` or ``optim.gradient_accumulation_steps`` (-1) from the global batch."""
        resolve_batching(self, data_parallel_world_size)


def resolve_batching(cfg: Any, dp: int) -> None:
    target = cfg.optim.global_batch_size
    ga = int(cfg.optim.gradient_accumulation_steps)
    mb = int(cfg.data.batch_size)
    if target is None:
        if ga == -1:
            raise ValueError("`optim.gradient_accumulation_steps=-1` requires `optim.global_batch_size`.")
        if mb == -1:
            raise ValueError("`data.batch_size=-1` requires `optim.global_batch_size`.")
        return
    if mb == -1 and ga == -1:
        raise ValueError("`optim.global_batch_size` cannot infer both `data.batch_size` and "
                         "`optim.gradient_accumulation_steps` at the same time.")
    if mb == -1:
        div = int(dp) * ga
        if div <= 0 or target % div:
            raise ValueError("`data.batch_size` cannot be inferred exactly: `optim.global_batch_size` must be "
                             "divisible by `data_parallel_world_size * optim.gradient_accumulation_steps`.")
        cfg.data.batch_size = mb = target // div
    elif ga == -1:
        div = int(dp) * mb
        if div <= 0 or target % div:
            raise ValueError("`optim.gradient_accumulation_steps` cannot be inferred exactly: "
                             "`optim.global_batch_size` must be divisible by `data_parallel_world_size * data.batch_size`.")
        cfg.optim.gradient_accumulation_steps = ga = target // div
    if int(dp) * mb * ga != target:
        raise ValueError("`optim.global_batch_size` does not match the configured batching: expected "
                         f"{int(dp) * mb * ga} from `data_parallel_world_size * data.batch_size * "
                         "optim.gradient_accumulation_steps`.")
