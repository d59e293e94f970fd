"""Megatron-style tensor / sequence parallelism via DTensor parallel styles
(reference: mvp_engine/distributed/tp.py:23-201).

The top-level model class declares ``TP_MODULE_CONFIG = {RuntimeClassName:
{child: "col" | "row"}}`` (plus ``SEQUENCE_PARALLEL_MODULE_CONFIG`` with
``"sequence"`` entries and ``SEQUENCE_PARALLEL_SEQUENCE_DIM``) and optional
``TP_MODULE_POSTPROCESSORS``.  Under sequence parallelism "col" takes a
sequence-sharded input and "row" produces a sequence-sharded output, so the
boundary collectives are all-gather in and reduce-scatter out.  The fused
NVLink versions of those two boundaries live in
:mod:`mvp_engine.parallel.tensor_parallel`.
"""

from __future__ import annotations

from typing import Any, Callable

import torch.nn as nn
from torch.distributed.tensor import Shard
from torch.distributed.tensor.parallel import (ColwiseParallel, ParallelStyle, RowwiseParallel, SequenceParallel,
                                               parallelize_module)

from ..utils.log import logger

TPModulePostprocessor = Callable[[nn.Module, Any], None]


def build_tp_plan(plan_cfg: object, sequence_parallel: bool = False, sequence_dim: int = 1) -> dict[str, ParallelStyle]:
    if not isinstance(plan_cfg, dict):
        raise TypeError(f"Unsupported TP plan config type: {type(plan_cfg)}")
    allowed = ("col", "row", "sequence") if sequence_parallel else ("col", "row")
    plan: dict[str, ParallelStyle] = {}
    for child, mode in plan_cfg.items():
        if not isinstance(mode, str):
            raise TypeError(f"TP mode for {child} must be str, got {type(mode)}.")
        mode = mode.lower()
        if mode not in allowed:
            raise ValueError(f"Unknown TP mode '{mode}' for {child}. Expected one of {allowed}.")
        if mode == "sequence":
            plan[child] = SequenceParallel(sequence_dim=sequence_dim, use_local_output=True)
        elif mode == "col":
            plan[child] = ColwiseParallel(input_layouts=Shard(sequence_dim)) if sequence_parallel else ColwiseParallel()
        else:
            plan[child] = RowwiseParallel(output_layouts=Shard(sequence_dim)) if sequence_parallel else RowwiseParallel()
    return plan


def _class_attr(model: nn.Module, name: str, required: bool, kind: type) -> Any:
    cls = type(model)
    if not hasattr(cls, name) or getattr(cls, name) is None:
        if required:
            raise AttributeError(f"{cls.__name__} does not define class attribute '{name}'. "
                                 "Please provide TP module plan via model class attribute.")
        return kind()
    val = getattr(cls, name)
    if not isinstance(val, kind):
        raise TypeError(f"{cls.__name__}.{name} must be {kind.__name__}, got {type(val)}.")
    return val


def merge_tp_configs(tp: dict, sp: dict) -> dict:
    out = dict(tp)
    for name, plan in sp.items():
        if name not in out:
            out[name] = plan
        elif isinstance(out[name], dict) and isinstance(plan, dict):
            out[name] = {**out[name], **plan}
        else:
            raise TypeError(f"Cannot merge TP and sequence-parallel plans for {name}: both plans must be dicts.")
    return out


def parallelize_model_with_tensor_parallel(model: nn.Module, tp_mesh, sequence_parallel: bool = False) -> None:
    config = _class_attr(model, "TP_MODULE_CONFIG", True, dict)
    post = _class_attr(model, "TP_MODULE_POSTPROCESSORS", False, dict)
    for k, fn in post.items():
        if not callable(fn):
            raise TypeError(f"{type(model).__name__}.TP_MODULE_POSTPROCESSORS[{k!r}] must be callable, got {type(fn)}.")
    seq_dim = 1
    if sequence_parallel:
        seq_dim = getattr(type(model), "SEQUENCE_PARALLEL_SEQUENCE_DIM", 1)
        if not isinstance(seq_dim, int):
            raise TypeError(f"{type(model).__name__}.SEQUENCE_PARALLEL_SEQUENCE_DIM must be int, got {type(seq_dim)}.")
        config = merge_tp_configs(config, _class_attr(model, "SEQUENCE_PARALLEL_MODULE_CONFIG", False, dict))
    counts: dict[str, int] = {}
    done: set[int] = set()
    for path, mod in sorted(model.named_modules(), key=lambda t: t[0].count("."), reverse=True):
        cls = type(mod).__name__
        if id(mod) in done or cls not in config:
            continue
        plan = build_tp_plan(config[cls], sequence_parallel, seq_dim)
        if not plan:
            continue
        parallelize_module(mod, tp_mesh, plan)
        if cls in post:
            post[cls](mod, tp_mesh)
        counts[cls] = counts.get(cls, 0) + 1
        done.add(id(mod))
    logger.info("Tensor Parallel Sharding: " + ", ".join(f"{c} x{n}" for c, n in sorted(counts.items())))
