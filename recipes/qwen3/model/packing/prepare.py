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


def build_packed_text_position_ids(input_ids: torch.Tensor, pack_segment_ids: torch.Tensor) -> torch.Tensor:
    """Position ids that restart at 0 in every packed document of every row; padding (segment id 0) gets 0."""
    from mvp_engine.kit.llm.data.collator import varlen_metadata

    _, _, pos = varlen_metadata(pack_segment_ids.detach().cpu())
    pos = pos.view(input_ids.shape).to(input_ids.device)
    return torch.where(pack_segment_ids.to(input_ids.device) > 0, pos, torch.zeros_like(pos))


def build_packed_fa2_varlen_kwargs(pack_segment_ids: torch.Tensor) -> dict[str, Any]:
    """Varlen attention arguments (``cu_seq_lens_q/k`` int32 over the flattened rows, ``max_length_q/k``)
    from ``[B, T]`` segment ids; a row's zero-padding suffix counts as one more document.  Rows must hold
    at least one real token and pad only at the end."""
    if pack_segment_ids.ndim != 2:
        raise ValueError(f"expected [batch, tokens] pack_segment_ids, got shape {tuple(pack_segment_ids.shape)}")
    from mvp_engine.kit.llm.data.collator import varlen_metadata

    real = pack_segment_ids.ne(0)
    if real.shape[1] and not bool(real[:, 0].all()):
        raise ValueError("every packed row needs at least one non-padding token, at its start")
    if bool((real[:, 1:] & ~real[:, :-1]).any()):
        raise ValueError("packed rows may pad only with one zero-valued suffix")
    cu, longest, _ = varlen_metadata(pack_segment_ids.detach().cpu())
    cu = cu.to(pack_segment_ids.device)
    return {"cu_seq_lens_q": cu, "cu_seq_lens_k": cu, "max_length_q": longest, "max_length_k": longest}
