"""Declarative specs of a multimodal data pipeline (reference: mvp_engine/kit/mllm/data/spec.py:14-161)."""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True, slots=True)
class MLLMSourceSpec:
    dataset_path: str
    dataset_source: str = "lance"
    ref_columns: tuple[str, ...] = ("images",)
    seed: int = 42
    resample: bool = True
    resolve_refs: bool = True

    def __post_init__(self) -> None:
        if not self.dataset_path:
            raise ValueError("MLLMSourceSpec.dataset_path must not be empty.")
        object.__setattr__(self, "ref_columns", tuple(self.ref_columns))


@dataclass(frozen=True, slots=True)
class MLLMSampleSpec:
    schema_handler: Any
    media_handler: Any
    tokenization_handler: Any


@dataclass(frozen=True, slots=True)
class MLLMPackingSpec:
    max_seq_len: int
    algorithm: str = "multi_pack"
    selection_strategy: str = "best_fit"
    open_pack_limit: int = 8
    buffer_size: int = 64
    block_causal: bool = True
    assembler_cls: type[Any] | None = None

    def __post_init__(self) -> None:
        if self.max_seq_len <= 0:
            raise ValueError("MLLMPackingSpec.max_seq_len must be positive.")
        if self.algorithm not in ("multi_pack", "packed"):
            raise ValueError("MLLMPackingSpec.algorithm must be 'multi_pack' or 'packed'.")
        if self.selection_strategy not in ("random", "best_fit"):
            raise ValueError("MLLMPackingSpec.selection_strategy must be one of random/best_fit.")
        if self.open_pack_limit <= 0:
            raise ValueError("MLLMPackingSpec.open_pack_limit must be positive.")
        if self.buffer_size < 0:
            raise ValueError("MLLMPackingSpec.buffer_size must be non-negative.")


@dataclass(frozen=True, slots=True)
class MLLMLoaderSpec:
    batch_size: int
    num_workers: int = 0
    pin_memory: bool | None = None
    persistent_workers: bool = False
    multiprocessing_context: str = "spawn"
    drop_last: bool = True

    def __post_init__(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("MLLMLoaderSpec.batch_size must be positive.")
        if self.num_workers < 0:
            raise ValueError("MLLMLoaderSpec.num_workers must be non-negative.")


@dataclass(frozen=True, slots=True)
class MLLMDistributionSpec:
    device_mesh: object | None = None
    dp_dims: str | Sequence[str] | None = None


@dataclass(frozen=True, slots=True)
class MLLMDataSpec:
    source: MLLMSourceSpec
    sample: MLLMSampleSpec
    packing: MLLMPackingSpec
    loader: MLLMLoaderSpec
    distribution: MLLMDistributionSpec | None = None
