"""Collated packed batch -> Qwen3-VL model inputs (reference: recipes/qwen3_vl/model/packing/prepare.py:11-95).

Everything here is host work on the CPU batch: 3-D M-RoPE position ids,
varlen ``cu_seq_lens_q`` / ``max_length_q`` over the packed documents (the
engine's attention consumes these, never a dense mask), and the vision
tower's per-image metadata (rotary angles, position-embedding interpolation
taps, per-image cu_seqlens).  The engine then copies the whole batch to the
GPU asynchronously from pinned memory.
"""

from __future__ import annotations

from typing import Any

import torch

from mvp_engine.kit.llm.data.collator import varlen_metadata

from .qwen3_vl import build_qwen3_vl_packed_position_ids

_DROP = ("source_sample_num", "num_input_tokens", "num_loss_tokens", "num_source_samples", "attention_mask")


def build_packed_varlen_kwargs(pack_segment_ids: torch.Tensor) -> dict[str, Any]:
    """cu_seqlens over the packed documents of all rows (padding suffix = one extra document)."""
    cu, mx, _ = varlen_metadata(pack_segment_ids.detach().cpu())
    return {"cu_seq_lens_q": cu, "cu_seq_lens_k": cu, "max_length_q": mx, "max_length_k": mx}


def prepare_packed_model_inputs(batch: dict[str, Any], *, model_config: Any, visual: Any = None,
                                attn_implementation: str | None = None,
                                mask_dtype: torch.dtype = torch.float32) -> dict[str, Any]:
    seg = batch.get("pack_segment_ids")
    if seg is None:
        raise ValueError("Packed Qwen3-VL batches must include pack_segment_ids.")
    out = {k: v for k, v in batch.items() if k not in _DROP}
    grid = out.get("image_grid_thw")
    out["position_ids"] = build_qwen3_vl_packed_position_ids(input_ids=out["input_ids"], pack_segment_ids=seg,
                                                             image_grid_thw=grid, model_config=model_config)
    out.update(build_packed_varlen_kwargs(seg))
    if visual is not None and grid is not None and grid.numel():
        out["vision_meta"] = visual.vision_metadata(grid.detach().cpu())
    return out


def build_packed_fa2_varlen_kwargs(pack_segment_ids: torch.Tensor) -> dict[str, Any]:
    """The reference's name for the varlen arguments of ``[B, T]`` segment ids (validated; see the Qwen3
    recipe's helper of the same name)."""
    from recipes.qwen3.model.packing.prepare import build_packed_fa2_varlen_kwargs as build

    return build(pack_segment_ids)


__all__ = ["build_packed_fa2_varlen_kwargs", "build_packed_varlen_kwargs", "prepare_packed_model_inputs"]
