"""Model families: Qwen3 (dense decoder), Qwen3-VL (vision tower + M-RoPE decoder), ViT
classifier, MagicTransformer."""

from __future__ import annotations

from typing import Any

import torch


def build_causal_lm(name_or_path: str, *, seed: int | None = 0, dtype: torch.dtype = torch.float32,
                    device: Any = None, **overrides: Any):
    """Resolve a model family from a preset name / local config and build it randomly initialised."""
    import json
    import os

    model_type = None
    cfg_file = os.path.join(name_or_path, "config.json")
    if os.path.isdir(name_or_path) and os.path.exists(cfg_file):
        with open(cfg_file) as f:
            model_type = json.load(f).get("model_type")
    lname = name_or_path.lower()
    if model_type in ("qwen3_vl",) or "qwen3-vl" in lname or "qwen3_vl" in lname:
        from .qwen3_vl import build_qwen3_vl

        return build_qwen3_vl(name_or_path, seed=seed, dtype=dtype, device=device, **overrides)
    from .qwen3 import build_qwen3

    return build_qwen3(name_or_path, seed=seed, dtype=dtype, device=device, **overrides)
