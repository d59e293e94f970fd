"""Magic Transformer config (reference: recipes/magic_transformer/configs/schema.py:8-50); adds
``model.routed_positions`` (see the model docstring)."""

from __future__ import annotations

from typing import Literal

from pydantic import BaseModel, ConfigDict, Field

from mvp_engine.config.schema import BaseEngineConfig, BaseOptimConfig


class MagicTransformerDataConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    fake_train_size: int = Field(128, ge=1)
    fake_eval_size: int = Field(32, ge=1)
    seq_len: int = Field(16, ge=2)
    vocab_size: int = Field(1024, ge=2)
    batch_size: int = Field(8, ge=1)
    num_workers: int = Field(0, ge=0)


class MagicTransformerModelConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="forbid")

    vocab_size: int = Field(1024, ge=2)
    max_seq_len: int = Field(16, ge=2)
    d_model: int = Field(128, ge=1)
    n_heads: int = Field(4, ge=1)
    n_kv_heads: int = Field(2, ge=1)
    n_layers: int = Field(4, ge=2)
    dropout: float = Field(0.0, ge=0.0, le=1.0)
    rope_base: float = Field(10000.0, gt=0.0)
    mod_top_k_ratio: float = Field(0.5, gt=0.0, le=1.0)
    dual_stream: bool = True
    router_ema_decay: float = Field(0.9, ge=0.0, le=1.0)
    routed_positions: Literal["compacted", "original"] = "compacted"


class MagicTransformerConfig(BaseEngineConfig):
    model_config = ConfigDict(frozen=False, extra="allow")

    data: MagicTransformerDataConfig = Field(default_factory=MagicTransformerDataConfig)
    model: MagicTransformerModelConfig = Field(default_factory=MagicTransformerModelConfig)
    optim: BaseOptimConfig = Field(default_factory=BaseOptimConfig)
