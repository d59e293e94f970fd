"""Drop-with-reason guards at each pipeline boundary (reference: mvp_engine/kit/llm/data/guard.py:27-167)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Iterable

import torch

from ....data import Assembler, stable_fingerprint
from ....utils.log import simple_info
from .sample import LLMSample
from .schema import LLMPretrainTextSchemaHandler, LLMSchemaHandler


@dataclass(frozen=True, slots=True)
class CheckResult:
    is_valid: bool
    reason: str | None = None


class LLMGuard(Assembler):
    def __init__(self, assemble_context: Any = None, *, verbose: bool = True) -> None:
        self.verbose = bool(verbose)
        self.dropped: dict[str, int] = {}

    def check(self, sample: Any) -> CheckResult:
        raise NotImplementedError

    def push(self, sample: Any) -> Iterable[Any]:
        res = self.check(sample)
        if res.is_valid:
            return [sample]
        reason = res.reason or "unknown"
        self.dropped[reason] = self.dropped.get(reason, 0) + 1
        if self.verbose:
            simple_info(f"Data guard skip: reason={reason} sample={self._info(sample)}", level="warning")
        return []

    @staticmethod
    def _info(sample: Any) -> Any:
        if isinstance(sample, LLMSample):
            sample = sample._raw
        if isinstance(sample, dict):
            return {k: sample[k] for k in ("id", "source", "__source__", "__key__", "__global_index__") if k in sample}
        text = repr(sample)
        return text[:200]


class LLMRawRowGuard(LLMGuard):
    def __init__(self, assemble_context: Any = None, *, schema_handler: LLMSchemaHandler | None = None,
                 verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.schema_handler = schema_handler or LLMPretrainTextSchemaHandler()

    def check(self, sample: Any) -> CheckResult:
        if not isinstance(sample, dict):
            return CheckResult(False, "raw.not_dict")
        reason = self.schema_handler.check_row(sample)
        return CheckResult(reason is None, reason)

    def fingerprint(self) -> str:
        return stable_fingerprint({"kind": type(self).__name__, "schema_handler": repr(self.schema_handler)})


class LLMSampleGuard(LLMGuard):
    def check(self, sample: Any) -> CheckResult:
        if not isinstance(sample, LLMSample):
            return CheckResult(False, "sample.invalid_type")
        sample.tokenize()
        if sample.token_length <= 0:
            return CheckResult(False, "sample.empty_tokens")
        ign = sample.tokenization_handler.ignore_index
        if all(lab == ign for lab in sample.labels):
            return CheckResult(False, "sample.no_supervised_tokens")
        return CheckResult(True)


class LLMModelInputGuard(LLMGuard):
    def __init__(self, assemble_context: Any = None, *, ignore_index: int = -100, verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.ignore_index = int(ignore_index)

    def check(self, sample: Any) -> CheckResult:
        if not isinstance(sample, dict):
            return CheckResult(False, "model_input.not_dict")
        for key in ("input_ids", "attention_mask", "labels", "pack_segment_ids"):
            v = sample.get(key)
            if not isinstance(v, torch.Tensor) or v.ndim != 1 or v.numel() == 0:
                return CheckResult(False, f"model_input.invalid_{key}")
        n = sample["input_ids"].shape
        if any(sample[k].shape != n for k in ("attention_mask", "labels", "pack_segment_ids")):
            return CheckResult(False, "model_input.shape_mismatch")
        if "position_ids" in sample and sample["position_ids"].shape != n:
            return CheckResult(False, "model_input.shape_mismatch")
        shifted = torch.nn.functional.pad(sample["labels"], (0, 1), value=self.ignore_index)[1:]
        if not bool(shifted.ne(self.ignore_index).any()):
            return CheckResult(False, "model_input.no_supervised_tokens")
        return CheckResult(True)
