"""Multimodal data guards: the LLM guards' rule tables plus image checks, and the text-only batch guard.

Public names and drop reasons of the reference's ``mvp_engine/kit/mllm/data/guard.py:30-452``.
"""

from __future__ import annotations

from typing import Any, Mapping, Sequence

import torch

from ...llm.data.guard import CheckResult, LLMGuard, Rule, _bad_vector
from .sample import MLLMSample


class MLLMGuard(LLMGuard):
    """Rule-table guard (see :class:`~mvp_engine.kit.llm.data.guard.LLMGuard`) for multimodal items."""


class MLLMRawRowGuard(MLLMGuard):
    """Raw rows: dicts whose ``images`` (if any) is a list, accepted by the schema handler."""

    def __init__(self, assemble_context: Any = None, *, schema_handler=None, verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.schema_handler = schema_handler

    def rules(self) -> Sequence[Rule]:
        return (("raw.not_dict", lambda row: not isinstance(row, dict)),
                ("raw.invalid_images", lambda row: row.get("images") is not None
                 and not isinstance(row["images"], (list, tuple))))

    def check(self, sample: Any) -> CheckResult:
        verdict = super().check(sample)
        if not verdict.is_valid or self.schema_handler is None:
            return verdict
        reason = self.schema_handler.check_row(sample)  # the handler names its own reason
        return CheckResult(reason is None, reason)


def _mllm_unsupervised(sample: MLLMSample) -> bool:
    ignore = sample.tokenization_handler.ignore_index
    return all(lab == ignore for lab in sample.labels)


class MLLMSampleGuard(MLLMGuard):
    """Tokenised samples: non-empty, with at least one supervised label."""

    def rules(self) -> Sequence[Rule]:
        return (("sample.invalid_type", lambda s: not isinstance(s, MLLMSample)),
                ("sample.empty_tokens", lambda s: s.tokenize().token_length <= 0),
                ("sample.no_supervised_tokens", _mllm_unsupervised))


def _image_tokens_disagree(item: dict, image_token_id: int, merge_size: int) -> bool:
    """The number of image placeholder tokens differs from the merged patch count of the images."""
    placeholders = int(item["input_ids"].eq(image_token_id).sum())
    merged = int(item["image_grid_thw"].prod(-1).sum()) // merge_size ** 2
    return placeholders != merged


class MLLMModelInputGuard(MLLMGuard):
    """Collated multimodal inputs: 1-D non-empty tensors, image placeholders matching the images'
    merged patches, some supervised label after the shift."""

    def __init__(self, assemble_context: Any = None, *, ignore_index: int = -100, image_token_id: int | None = None,
                 merge_size: int = 2, verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.ignore_index = int(ignore_index)
        self.image_token_id = image_token_id
        self.merge_size = merge_size

    def rules(self) -> Sequence[Rule]:
        vectors = ("input_ids", "attention_mask", "labels", "pack_segment_ids")
        token_id = self.image_token_id
        return (
            ("model_input.empty", lambda x: not isinstance(x, dict) or bool(x.get("__empty__"))),
            *((f"model_input.invalid_{k}", _bad_vector(k)) for k in vectors),
            ("model_input.image_token_mismatch", lambda x: token_id is not None and "image_grid_thw" in x
             and _image_tokens_disagree(x, token_id, self.merge_size)),
            ("model_input.no_supervised_tokens", lambda x: not bool(x["labels"][1:].ne(self.ignore_index).any())),
        )


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
