"""Packed-batch -> model inputs (reference: recipes/qwen3/model/packing/prepare.py:8-91).

The varlen metadata (``cu_seq_lens_q``, ``max_length_q``, per-document
``position_ids``) is computed by the collator on the CPU; this step only
forwards the fields the model consumes and, for segment-free batches (plain
causal streams), falls back to one document per row.
"""

from __future__ import annotations

from typing import Any

import torch


def prepare_packed_model_inputs(batch: dict[str, Any], *, attn_implementation: str | None = None,
                                mask_dtype: torch.dtype = torch.float32) -> dict[str, Any]:
    out = dict(batch)
    out.pop("attention_mask", None)  # document structure travels as cu_seqlens, never as a mask
    if "cu_seq_lens_q" not in out:
        from mvp_engine.kit.llm.data.collator import varlen_metadata

        seg = out.get("pack_segment_ids")
        if seg is None:
            seg = torch.ones_like(out["input_ids"])
        cu, mx, pos = varlen_metadata(seg.cpu())
        out["cu_seq_lens_q"] = cu.to(out["input_ids"].device)
        out["max_length_q"] = mx
        out.setdefault("position_ids", pos.to(out["input_ids"].device))
    return out
