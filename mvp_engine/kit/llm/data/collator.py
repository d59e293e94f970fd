"""Batch collation with token accounting (reference: mvp_engine/kit/llm/data/collator.py:11-62).

Besides the reference fields this collator also computes, on the CPU at
collate time, the flat varlen metadata the packed-attention kernels consume
(``cu_seq_lens_q``/``max_length_q`` and per-document ``position_ids``), so the
training step needs no ``.item()`` host syncs to build it.
"""

from __future__ import annotations

from typing import Any

import torch
from torch.nn.utils.rnn import pad_sequence

from .types import ModelInputs


def varlen_metadata(pack_segment_ids: torch.Tensor) -> tuple[torch.Tensor, int, torch.Tensor]:
    """(cu_seqlens int32 over the flattened batch, max doc length, per-document positions)."""
    seg = pack_segment_ids.reshape(pack_segment_ids.shape[0], -1)
    B, T = seg.shape
    flat = seg.reshape(-1)
    start = torch.ones_like(flat, dtype=torch.bool)
    start[1:] = flat[1:] != flat[:-1]
    start[::T] = True
    idx = torch.nonzero(start).reshape(-1)
    cu = torch.cat([idx, torch.tensor([flat.numel()])]).to(torch.int32)
    lens = cu[1:] - cu[:-1]
    doc = torch.cumsum(start.long(), 0) - 1
    pos = torch.arange(flat.numel()) - cu[doc].long()
    return cu, int(lens.max()) if lens.numel() else 0, pos.view(B, T)


class LLMBatchCollator:
    def __init__(self, pad_token_id: int, *, ignore_index: int = -100, varlen: bool = True) -> None:
        self.pad_token_id = int(pad_token_id)
        self.ignore_index = int(ignore_index)
        self.varlen = varlen

    def __call__(self, batch: list[dict[str, Any]]) -> ModelInputs:
        if not all("pack_segment_ids" in s for s in batch):
            raise ValueError("Packed LLM samples must include pack_segment_ids.")
        if not all("source_sample_num" in s for s in batch):
            raise ValueError("Packed LLM samples must include source_sample_num.")
        ids = pad_sequence([s["input_ids"] for s in batch], batch_first=True, padding_value=self.pad_token_id)
        am = pad_sequence([s["attention_mask"] for s in batch], batch_first=True, padding_value=0)
        labels = pad_sequence([s["labels"] for s in batch], batch_first=True, padding_value=self.ignore_index)
        seg = pad_sequence([s["pack_segment_ids"] for s in batch], batch_first=True, padding_value=0)
        nsrc = torch.tensor([int(s["source_sample_num"]) for s in batch], dtype=torch.long)
        out: dict[str, Any] = {"input_ids": ids, "attention_mask": am, "labels": labels, "pack_segment_ids": seg,
                               "source_sample_num": nsrc}
        if all("position_ids" in s for s in batch):
            out["position_ids"] = pad_sequence([s["position_ids"] for s in batch], batch_first=True, padding_value=0)
        n_in = am.sum(-1)
        shifted = torch.nn.functional.pad(labels, (0, 1), value=self.ignore_index)[..., 1:]
        n_loss = shifted.ne(self.ignore_index).sum(-1)
        out["num_input_tokens"] = n_in
        out["num_loss_tokens"] = n_loss
        out["num_source_samples"] = nsrc.clone()
        out["total_tokens"] = int(n_in.sum())
        out["effective_tokens"] = int(n_loss.sum())
        # Logical attention pairs (sum of squared document lengths) for FLOPs accounting,
        # computed here so the training step never syncs to count them.
        pairs = 0
        for row in seg:
            ids = row[row > 0]
            if ids.numel():
                pairs += int(torch.bincount(ids).pow(2).sum())
        out["attention_token_pairs"] = pairs
        if self.varlen:
            cu, mx, pos = varlen_metadata(seg)
            out["cu_seq_lens_q"] = cu
            out["cu_seq_lens_k"] = cu
            out["max_length_q"] = mx
            out["max_length_k"] = mx
            if "position_ids" not in out:
                out["position_ids"] = pos
        return out
