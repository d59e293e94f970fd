"""Multimodal data guards (reference: mvp_engine/kit/mllm/data/guard.py:30-452)."""

from __future__ import annotations

from typing import Any, Mapping, Sequence

import torch

from ...llm.data.guard import CheckResult, LLMGuard
from .sample import MLLMSample


class MLLMGuard(LLMGuard):
    pass


class MLLMRawRowGuard(MLLMGuard):
    def __init__(self, assemble_context: Any = None, *, schema_handler=None, verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.schema_handler = schema_handler

    def check(self, sample: Any) -> CheckResult:
        if not isinstance(sample, dict):
            return CheckResult(False, "raw.not_dict")
        imgs = sample.get("images")
        if imgs is not None and not isinstance(imgs, (list, tuple)):
            return CheckResult(False, "raw.invalid_images")
        if self.schema_handler is not None:
            reason = self.schema_handler.check_row(sample)
            if reason is not None:
                return CheckResult(False, reason)
        return CheckResult(True)


class MLLMSampleGuard(MLLMGuard):
    def check(self, sample: Any) -> CheckResult:
        if not isinstance(sample, MLLMSample):
            return CheckResult(False, "sample.invalid_type")
        sample.tokenize()
        if sample.token_length <= 0:
            return CheckResult(False, "sample.empty_tokens")
        ign = sample.spec.tokenization_handler.ignore_index
        if all(lab == ign for lab in sample.labels):
            return CheckResult(False, "sample.no_supervised_tokens")
        return CheckResult(True)


class MLLMModelInputGuard(MLLMGuard):
    def __init__(self, assemble_context: Any = None, *, ignore_index: int = -100, image_token_id: int | None = None,
                 merge_size: int = 2, verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.ignore_index = int(ignore_index)
        self.image_token_id = image_token_id
        self.merge_size = merge_size

    def check(self, sample: Any) -> CheckResult:
        if not isinstance(sample, dict) or sample.get("__empty__"):
            return CheckResult(False, "model_input.empty")
        for key in ("input_ids", "attention_mask", "labels", "pack_segment_ids"):
            v = sample.get(key)
            if not isinstance(v, torch.Tensor) or v.ndim != 1 or v.numel() == 0:
                return CheckResult(False, f"model_input.invalid_{key}")
        if self.image_token_id is not None and "image_grid_thw" in sample:
            n_tok = int((sample["input_ids"] == self.image_token_id).sum())
            n_feat = int(sample["image_grid_thw"].prod(-1).sum()) // self.merge_size ** 2
            if n_tok != n_feat:
                return CheckResult(False, "model_input.image_token_mismatch")
        shifted = torch.nn.functional.pad(sample["labels"], (0, 1), value=self.ignore_index)[1:]
        if not bool(shifted.ne(self.ignore_index).any()):
            return CheckResult(False, "model_input.no_supervised_tokens")
        return CheckResult(True)


class MLLMTextOnlyBatchGuard:
    """Give a text-only batch one tiny dummy image (isolated segment, ignored labels) so the
    vision tower runs on every rank of every step (sharded parameters must all be used)."""

    def __init__(self, *, dummy_inputs: Mapping[str, torch.Tensor], media_keys: Sequence[str], pad_token_id: int,
                 ignore_index: int = -100) -> None:
        self.dummy = {k: (v.detach().clone() if isinstance(v, torch.Tensor) else v) for k, v in dummy_inputs.items()}
        self.media_keys = tuple(media_keys)
        self.pad_token_id = int(pad_token_id)
        self.ignore_index = int(ignore_index)
        missing = {"input_ids", "attention_mask", *self.media_keys} - set(self.dummy)
        if missing:
            raise ValueError(f"Dummy media inputs are missing keys: {sorted(missing)}")

    def __call__(self, batch: dict[str, Any]) -> dict[str, Any]:
        if any(isinstance(batch.get(k), torch.Tensor) and batch[k].numel() > 0 for k in self.media_keys):
            return batch
        ids = batch["input_ids"]
        B, L = ids.shape
        d_ids = self.dummy["input_ids"].to(ids)
        n = d_ids.numel()
        lens = batch["attention_mask"].sum(-1).long()
        out_len = max(L, int(lens[0]) + n)
        new = dict(batch)

        def grow(x, fill):
            y = torch.full((B, out_len), fill, dtype=x.dtype, device=x.device)
            y[:, :L] = x
            return y

        new["input_ids"] = grow(ids, self.pad_token_id)
        new["attention_mask"] = grow(batch["attention_mask"], 0)
        new["labels"] = grow(batch["labels"], self.ignore_index)
        new["pack_segment_ids"] = grow(batch["pack_segment_ids"], 0)
        s = int(lens[0])
        seg_id = int(new["pack_segment_ids"][0, :s].max()) + 1
        new["input_ids"][0, s:s + n] = d_ids
        new["attention_mask"][0, s:s + n] = 1
        new["labels"][0, s:s + n] = self.ignore_index
        new["pack_segment_ids"][0, s:s + n] = seg_id
        for k in self.media_keys:
            new[k] = self.dummy[k].clone()
        new["num_input_tokens"] = new["attention_mask"].sum(-1)
        new["total_tokens"] = int(new["num_input_tokens"].sum())
        new.pop("position_ids", None)
        new.pop("cu_seq_lens_q", None)
        return new

    def fingerprint(self) -> str:
        from ....data import stable_fingerprint

        return stable_fingerprint({"kind": type(self).__name__, "keys": self.media_keys})
