"""Multimodal batch collation (reference: mvp_engine/kit/mllm/data/collator.py:11-89).

Pads token fields, concatenates media tensors through the media handler and
adds token counts (shifted labels) like the text collator, plus the
``attention_token_pairs`` used for FLOPs accounting.
"""

from __future__ import annotations

from typing import Any

import torch
from torch.nn.utils.rnn import pad_sequence


class MLLMBatchCollator:
    def __init__(self, *, pad_token_id: int, media_handler: Any = None, ignore_index: int = -100) -> None:
        self.pad_token_id = int(pad_token_id)
        self.media_handler = media_handler
        self.ignore_index = int(ignore_index)

    def __call__(self, batch: list[dict[str, Any]]) -> dict[str, Any]:
        ids = pad_sequence([b["input_ids"] for b in batch], batch_first=True, padding_value=self.pad_token_id)
        am = pad_sequence([b["attention_mask"] for b in batch], batch_first=True, padding_value=0)
        labels = pad_sequence([b["labels"] for b in batch], batch_first=True, padding_value=self.ignore_index)
        seg = pad_sequence([b["pack_segment_ids"] for b in batch], batch_first=True, padding_value=0)
        nsrc = torch.tensor([int(b.get("source_sample_num", 1)) for b in batch], dtype=torch.long)
        out: dict[str, Any] = {"input_ids": ids, "attention_mask": am, "labels": labels, "pack_segment_ids": seg,
                               "source_sample_num": nsrc}
        if self.media_handler is not None:
            out.update(self.media_handler.collate(batch))
        n_in = am.sum(-1)
        shifted = torch.nn.functional.pad(labels, (0, 1), value=self.ignore_index)[..., 1:]
        n_loss = shifted.ne(self.ignore_index).sum(-1)
        out.update({"num_input_tokens": n_in, "num_loss_tokens": n_loss, "num_source_samples": nsrc.clone(),
                    "total_tokens": int(n_in.sum()), "effective_tokens": int(n_loss.sum())})
        pairs = 0
        for row in seg:
            r = row[row > 0]
            if r.numel():
                pairs += int(torch.bincount(r).pow(2).sum())
        out["attention_token_pairs"] = pairs
        return out
