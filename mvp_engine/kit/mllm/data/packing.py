"""Streaming multi-pack packing (reference: mvp_engine/kit/mllm/data/packing.py:35-329).

Samples wait in a pending pool (at most ``buffer_size``) and are placed into
up to ``open_pack_limit`` open packs: ``best_fit`` chooses the open pack whose
remaining room is smallest but sufficient, ``random`` a random fitting one.
A pack that becomes exactly full is emitted; when nothing fits and no new pack
may open, or the pool overflows, the most-filled open pack is closed and
emitted.  ``finish`` drains everything.  Samples longer than ``max_seq_len``
raise.  ``algorithm="packed"`` emits each sample on its own.  State (open
packs, pending pool, RNG) is resumable.
"""

from __future__ import annotations

import random
from typing import Any, Iterable, Optional

import torch

from ....data import Assembler, stable_fingerprint
from .sample import MLLMPack, MLLMSample
from .spec import MLLMPackingSpec


class MLLMPackingAssembler(Assembler):
    def __init__(self, spec: MLLMPackingSpec, assemble_context: Any = None, *, seed: int = 0) -> None:
        self.spec = spec
        self.open: list[list[MLLMSample]] = []
        self.pending: list[MLLMSample] = []
        self.rng = random.Random(seed)

    def _room(self, pack: list[MLLMSample]) -> int:
        return self.spec.max_seq_len - sum(s.token_length for s in pack)

    def push(self, sample: MLLMSample) -> Iterable[MLLMPack]:
        n = sample.token_length
        if n <= 0:
            return []
        if n > self.spec.max_seq_len:
            raise ValueError(f"sample of {n} tokens exceeds max_seq_len={self.spec.max_seq_len}")
        if self.spec.algorithm == "packed":
            return [MLLMPack([sample])]
        self.pending.append(sample)
        out = self._assign()
        while len(self.pending) > self.spec.buffer_size:
            out.append(self._close_most_filled())
            out += self._assign()
        return out

    def _choose(self, n: int) -> Optional[int]:
        fits = [i for i, p in enumerate(self.open) if self._room(p) >= n]
        if not fits:
            return None
        if self.spec.selection_strategy == "random":
            return self.rng.choice(fits)
        return min(fits, key=lambda i: self._room(self.open[i]))

    def _assign(self) -> list[MLLMPack]:
        out: list[MLLMPack] = []
        still: list[MLLMSample] = []
        for s in self.pending:
            i = self._choose(s.token_length)
            if i is None and len(self.open) < self.spec.open_pack_limit:
                self.open.append([])
                i = len(self.open) - 1
            if i is None:
                still.append(s)
                continue
            self.open[i].append(s)
            if self._room(self.open[i]) == 0:
                out.append(MLLMPack(self.open.pop(i)))
        self.pending = still
        return out

    def _close_most_filled(self) -> MLLMPack:
        i = min(range(len(self.open)), key=lambda j: self._room(self.open[j]))
        return MLLMPack(self.open.pop(i))

    def finish(self, *, drop_last: bool = False) -> Iterable[MLLMPack]:
        out = []
        while self.pending:
            out += self._assign()
            if self.pending:
                out.append(self._close_most_filled())
        out += [MLLMPack(p) for p in self.open if p]
        self.open = []
        return out

    def state_dict(self) -> dict[str, object]:
        return {"open": [[s._raw for s in p] for p in self.open], "pending": [s._raw for s in self.pending],
                "rng": self.rng.getstate()}

    def load_state_dict(self, state: dict[str, object], sample_spec=None) -> None:
        if sample_spec is None:
            raise ValueError("MLLMPackingAssembler.load_state_dict needs the sample spec to rebuild samples")
        self.open = [[MLLMSample.from_row(r, sample_spec=sample_spec) for r in p] for p in state.get("open", [])]
        self.pending = [MLLMSample.from_row(r, sample_spec=sample_spec) for r in state.get("pending", [])]
        if "rng" in state:
            self.rng.setstate(state["rng"])

    def fingerprint(self) -> str:
        s = self.spec
        return stable_fingerprint({"max_seq_len": s.max_seq_len, "algorithm": s.algorithm,
                                   "selection": s.selection_strategy, "open": s.open_pack_limit,
                                   "buffer": s.buffer_size, "block_causal": s.block_causal})


def build_packed_block_causal_mask(pack_segment_ids: torch.Tensor, *, dtype: torch.dtype) -> torch.Tensor:
    from ...llm.data.packing import build_packed_block_causal_mask as _b

    return _b(pack_segment_ids, dtype=dtype)
