"""Pydantic v2 configuration schema (reference: mvp_engine/config/schema.py:8-128).

Same fields and validation as the reference, plus the B200 engine's
additions: ``parallel.mesh.context`` (context-parallel degree) and
``parallel.backend_kwargs.{impl, context_parallel, comm}`` selecting the
native data-parallel runtime, the context-parallel algorithm and whether the
fused NVLink kernels or plain NCCL carry the collectives.
"""

from __future__ import annotations

from typing import Literal, Optional

from pydantic import BaseModel, ConfigDict, Field, field_validator

from ..utils.tracing import TraceConfig


class BaseLogConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    interval: int = Field(20, ge=1)
    backends: list[Literal["terminal", "file", "wandb"]] = ["terminal", "file"]
    accumulation_size: Optional[int] = Field(None, ge=1)
    timer_window_size: int = Field(100, ge=1)


class BaseProjectConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    name: str = "mvp-engine"
    dir: str = "./outputs"


class BaseRuntimeInfo(BaseModel):
    model_config = ConfigDict(frozen=False)

    git_info: str = ""
    run_id: str = ""
    output_dir: str = ""
    world_size: int = 1
    hostname: str = ""
    python_version: str = ""
    torch_version: str = ""


class BaseMeshConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    replicate: int = 1
    shard: int = 8
    context: int = 1
    tensor: int = 1

    @field_validator("replicate", "shard", "context", "tensor")
    @classmethod
    def validate_mesh_dim(cls, v: int) -> int:
        if v == 0 or v < -1:
            raise ValueError("Mesh dimensions must be >= 1 or exactly -1")
        return v


class BaseMpPolicyConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    param_dtype: Literal["float32", "float16", "bfloat16"] = "bfloat16"
    reduce_dtype: Literal["float32", "float16", "bfloat16"] = "float32"
    output_dtype: Literal["float32", "float16", "bfloat16"] = "bfloat16"
    buffer_dtype: Literal["float32", "float16", "bfloat16"] = "bfloat16"


class BaseFSDP2Config(BaseModel):
    model_config = ConfigDict(frozen=False, extra="allow")

    reshard_after_forward: bool = True
    offload_policy: bool = False
    mp_policy: BaseMpPolicyConfig = Field(default_factory=BaseMpPolicyConfig)
    high_precision_modules: list[str] = []
    target_classes: list[str] = []


class BaseDDPConfig(BaseModel):
    model_config = ConfigDict(frozen=False, extra="allow")


class ContextParallelConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    impl: Literal["ring", "ulysses"] = "ring"


class CommConfig(BaseModel):
    """``fused``: collectives run in the engine's own NVLink kernels; else NCCL."""

    model_config = ConfigDict(frozen=False)

    fused: bool = True
    bucket_mb: int = Field(256, ge=1)


class BaseBackendKwargsConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    sequence_parallel: bool = False
    # "native": flat-buffer FSDP with native kernels (B200 path);
    # "torch": torch FSDP2 / DDP exactly as the reference wraps models.
    impl: Literal["native", "torch"] = "native"
    fsdp2: BaseFSDP2Config = Field(default_factory=BaseFSDP2Config)
    ddp: BaseDDPConfig = Field(default_factory=BaseDDPConfig)
    context_parallel: ContextParallelConfig = Field(default_factory=ContextParallelConfig)
    comm: CommConfig = Field(default_factory=CommConfig)
    # native runtime: free each decoder block's full weights after use and gather them again when needed
    # (FSDP2's reshard_after_forward).  None: keep them resident unless they would take more than a fifth
    # of the device's memory.
    reshard_after_forward: Optional[bool] = None


class BaseParallelConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    mesh: BaseMeshConfig = Field(default_factory=BaseMeshConfig)
    backend_kwargs: BaseBackendKwargsConfig = Field(default_factory=BaseBackendKwargsConfig)


class BaseOptimConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    lr: float = 1e-3
    weight_decay: float = 0.05
    gradient_accumulation_steps: int = Field(1, ge=1)
    mixed_precision: Literal["fp32", "fp16", "bf16"] = "bf16"
    warmup_ratio: float = Field(0.1, ge=0.0, le=1.0)
    clip_grad_norm: Optional[float] = 5.0


class BaseCheckpointConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    keep_n: int = Field(5, ge=1)
    interval: int = Field(5000, ge=1)
    hf_enable: bool = False


class BaseLoopConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    policy: Literal["iter", "epoch"] = "iter"
    total_steps: int = Field(10000, ge=1)


class BaseEngineConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    dev_mode: bool = False
    engine: str = "Engine"
    seed: int = 42
    deterministic: bool = False
    project: BaseProjectConfig = Field(default_factory=BaseProjectConfig)
    runtime: BaseRuntimeInfo = Field(default_factory=BaseRuntimeInfo)
    log: BaseLogConfig = Field(default_factory=BaseLogConfig)
    parallel: BaseParallelConfig = Field(default_factory=BaseParallelConfig)
    optim: BaseOptimConfig = Field(default_factory=BaseOptimConfig)
    loop: BaseLoopConfig = Field(default_factory=BaseLoopConfig)
    checkpoint: BaseCheckpointConfig = Field(default_factory=BaseCheckpointConfig)
    # NVTX ranges per phase / block and an opt-in torch.profiler window (all off by default)
    trace: TraceConfig = Field(default_factory=TraceConfig)
    # A checkpoint directory to resume from, or "latest": the newest complete checkpoint of this
    # project (none -> fresh start), for automatic restarts after a failure.
    resume: Optional[str] = None
