"""Sequential token-stream packing (reference: mvp_engine/kit/llm/data/packing.py:16-190).

Samples are concatenated in stream order and the stream is cut into
``max_seq_len`` packs.  ``isolate_attention`` numbers documents 1..n inside a
pack (``pack_segment_ids``; otherwise all ones, i.e. one causal stream),
``isolate_position_ids`` restarts positions at each document.  The state is
resumable (``state_dict``) and the configuration fingerprinted.
"""

from __future__ import annotations

from typing import Any, Iterable

import torch

from ....data import Assembler, stable_fingerprint
from .sample import LLMPack, LLMSample
from .spec import LLMPackingSpec


class LLMPackingAssembler(Assembler):
    def __init__(self, spec: LLMPackingSpec, assemble_context: Any = None) -> None:
        self.spec = spec
        self.pending_input_ids: list[int] = []
        self.pending_labels: list[int] = []
        self.pending_sample_ids: list[int] = []
        self.next_sample_id = 1
        self.pad_token_id: int | None = None
        self.ignore_index = -100

    def push(self, sample: LLMSample) -> Iterable[LLMPack]:
        n = sample.token_length
        if n <= 0:
            return []
        tok = sample.tokenization_handler.tokenizer
        if getattr(tok, "pad_token_id", None) is not None:
            self.pad_token_id = int(tok.pad_token_id)
        self.ignore_index = int(sample.tokenization_handler.ignore_index)
        sid = self.next_sample_id
        self.next_sample_id += 1
        self.pending_input_ids += sample.input_ids
        self.pending_labels += sample.labels
        self.pending_sample_ids += [sid] * n
        return self._drain()

    def finish(self, *, drop_last: bool = False) -> Iterable[LLMPack]:
        out = self._drain()
        if self.pending_input_ids and self.spec.tail_policy == "pad" and not drop_last:
            out.append(self._take(len(self.pending_input_ids), pad_to=self.spec.max_seq_len))
        self.pending_input_ids, self.pending_labels, self.pending_sample_ids = [], [], []
        return out

    def state_dict(self) -> dict[str, object]:
        return {"pending_input_ids": list(self.pending_input_ids), "pending_labels": list(self.pending_labels),
                "pending_sample_ids": list(self.pending_sample_ids), "next_sample_id": self.next_sample_id,
                "pad_token_id": self.pad_token_id, "ignore_index": self.ignore_index}

    def load_state_dict(self, state: dict[str, object]) -> None:
        self.pending_input_ids = list(state.get("pending_input_ids", []))
        self.pending_labels = list(state.get("pending_labels", []))
        self.pending_sample_ids = list(state.get("pending_sample_ids", []))
        self.next_sample_id = int(state.get("next_sample_id", 1))
        pad = state.get("pad_token_id")
        self.pad_token_id = int(pad) if pad is not None else None
        self.ignore_index = int(state.get("ignore_index", -100))

    def fingerprint(self) -> str:
        s = self.spec
        return stable_fingerprint({"max_seq_len": s.max_seq_len, "tail_policy": s.tail_policy,
                                   "isolate_attention": s.isolate_attention,
                                   "isolate_position_ids": s.isolate_position_ids})

    def _drain(self) -> list[LLMPack]:
        out = []
        while len(self.pending_input_ids) >= self.spec.max_seq_len:
            out.append(self._take(self.spec.max_seq_len))
        return out

    def _take(self, n: int, pad_to: int | None = None) -> LLMPack:
        ids, labels, sids = self.pending_input_ids[:n], self.pending_labels[:n], self.pending_sample_ids[:n]
        del self.pending_input_ids[:n], self.pending_labels[:n], self.pending_sample_ids[:n]
        pad = 0 if pad_to is None else pad_to - n
        if pad < 0:
            raise ValueError("Cannot pad a pack to a length shorter than its token count.")
        if pad:
            if self.pad_token_id is None:
                raise ValueError("Tokenizer must expose pad_token_id when LLMPackingSpec.tail_policy='pad'.")
            ids = ids + [self.pad_token_id] * pad
            labels = labels + [self.ignore_index] * pad
        seg, pos, cur, seg_no, p = [], [], None, 0, 0
        for s in sids:
            if s != cur:
                cur, seg_no, p = s, seg_no + 1, 0
            seg.append(seg_no if self.spec.isolate_attention else 1)
            pos.append(p)
            p += 1
        return LLMPack(input_ids=ids, labels=labels, attention_mask=[1] * len(sids) + [0] * pad,
                       pack_segment_ids=seg + [0] * pad, source_sample_num=len(set(sids)),
                       position_ids=(pos + [0] * pad) if self.spec.isolate_position_ids else None)


def build_packed_block_causal_mask(pack_segment_ids: torch.Tensor, *, dtype: torch.dtype) -> torch.Tensor:
    """Additive [B, 1, T, T] mask (0 allowed, dtype-min blocked) for eager / SDPA paths."""
    seg = pack_segment_ids
    same = seg.unsqueeze(-1) == seg.unsqueeze(-2)
    valid = (seg > 0).unsqueeze(-1) & (seg > 0).unsqueeze(-2)
    T = seg.shape[-1]
    causal = torch.ones(T, T, dtype=torch.bool, device=seg.device).tril()
    allowed = same & valid & causal
    mask = torch.zeros(allowed.shape, dtype=dtype, device=seg.device)
    mask.masked_fill_(~allowed, torch.finfo(dtype).min)
    return mask.unsqueeze(1)
