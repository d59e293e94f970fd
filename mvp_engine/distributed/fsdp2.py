"""torch FSDP2 wrapping with the reference's policy (reference: mvp_engine/distributed/fsdp2.py:50-176).

Every module whose class is in ``model._no_split_modules`` or ``target_classes``
is ``fully_shard``-ed deepest first, ``high_precision_modules`` keep fp32
params (only the reduce dtype of the default policy), ``ignore_modules``
outside wrapped subtrees are excluded, then the root is wrapped and an
optional ``APPLY_FSDP2_CUSTOM_PREFETCHING`` class hook runs.  This is the
library baseline path; the B200 path is :mod:`mvp_engine.parallel.fsdp`.
"""

from __future__ import annotations

from typing import Any, Callable, Optional

import torch
import torch.nn as nn
from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

from ..utils.log import logger


def _to_dtype(v: Any) -> Optional[torch.dtype]:
    if v is None or isinstance(v, torch.dtype):
        return v
    if isinstance(v, str) and hasattr(torch, v):
        return getattr(torch, v)
    raise ValueError(f"Unsupported dtype value: {v!r}")


def build_mp_policy(cfg: Any) -> Optional[MixedPrecisionPolicy]:
    if cfg is None or isinstance(cfg, MixedPrecisionPolicy):
        return cfg
    return MixedPrecisionPolicy(param_dtype=_to_dtype(cfg.get("param_dtype")),
                                reduce_dtype=_to_dtype(cfg.get("reduce_dtype")),
                                output_dtype=_to_dtype(cfg.get("output_dtype")),
                                cast_forward_inputs=cfg.get("cast_forward_inputs", True))


def _class_hook(model: nn.Module, name: str) -> Optional[Callable[[nn.Module], None]]:
    hook = getattr(type(model), name, None)
    if hook is None:
        return None
    if not callable(hook):
        raise TypeError(f"{type(model).__name__}.{name} must be callable, got {type(hook)}.")
    return hook


def parallelize_model_with_fsdp2(model: nn.Module, backend_kwargs: Optional[dict] = None) -> nn.Module:
    from ..patches import apply_all_patches

    apply_all_patches()  # recomputed FSDP2 modules must cast their inputs (whatever the entry point)
    kw = dict(backend_kwargs or {})
    targets = set(getattr(model, "_no_split_modules", []) or []) | set(kw.pop("target_classes", []) or [])
    hp_classes = set(kw.pop("high_precision_modules", []) or [])
    hp_policy = build_mp_policy(kw.pop("high_precision_mp_policy", None))
    ignore_classes = set(kw.pop("ignore_modules", []) or [])
    for k in ("reduce_dtype_override",):
        kw.pop(k, None)
    default_policy = build_mp_policy(kw.get("mp_policy"))
    kw["mp_policy"] = default_policy
    if hp_classes and hp_policy is None and isinstance(default_policy, MixedPrecisionPolicy):
        hp_policy = MixedPrecisionPolicy(param_dtype=None, reduce_dtype=default_policy.reduce_dtype,
                                         output_dtype=None, cast_forward_inputs=default_policy.cast_forward_inputs)
    wrapped: list[tuple[str, nn.Module, dict]] = []
    roots: set[str] = set()
    for fqn, mod in model.named_modules():
        cls = type(mod).__name__
        if cls in hp_classes:
            wrapped.append((fqn, mod, {**kw, "mp_policy": hp_policy} if hp_policy is not None else kw))
            roots.add(fqn)
        elif cls in targets:
            wrapped.append((fqn, mod, kw))
            roots.add(fqn)

    def inside(fqn: str) -> bool:
        return any(r == "" or fqn == r or fqn.startswith(r + ".") for r in roots)

    ignored: set[nn.Parameter] = set()
    for fqn, mod in model.named_modules():
        if fqn and not inside(fqn) and type(mod).__name__ in ignore_classes:
            ignored.update(mod.parameters(recurse=False))
    logger.info("FSDP2 Sharding: " + ", ".join(sorted(targets | hp_classes)))
    wrapped.sort(key=lambda t: t[0].count("."), reverse=True)
    for _, mod, skw in wrapped:
        fully_shard(mod, **skw)
    fully_shard(model, **kw, ignored_params=ignored or None)
    hook = _class_hook(model, "APPLY_FSDP2_CUSTOM_PREFETCHING")
    if hook is not None:
        logger.info(f"Applying custom FSDP2 prefetching on {type(model).__name__}...")
        hook(model)
    return model
