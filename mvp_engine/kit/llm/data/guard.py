"""Guards that drop invalid items at each boundary of the text pipeline, with a logged reason.

Public API of the reference's ``mvp_engine/kit/llm/data/guard.py:27-167`` (class names,
``check`` -> :class:`CheckResult`, the ``reason`` strings users grep logs for).

Each guard here is a list of *rules*: a rule is a reason string and a test that
returns True when the item must be dropped.  ``check`` returns the first rule
that fires.  Guards also count what they dropped per reason (``dropped``), so a
run can report how much data each boundary removed.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Iterable, Optional, Sequence

import torch

from ....data import Assembler, stable_fingerprint
from ....utils.log import simple_info
from .sample import LLMSample
from .schema import LLMPretrainTextSchemaHandler, LLMSchemaHandler

_INFO_KEYS = ("id", "source", "__source__", "__key__", "__global_index__")
Rule = tuple[str, Callable[[Any], bool]]


@dataclass(frozen=True)
class CheckResult:
    is_valid: bool
    reason: Optional[str] = None


class LLMGuard(Assembler):
    """Pass-through assembler that drops items failing any of :meth:`rules`."""

    def __init__(self, assemble_context: Any = None, *, verbose: bool = True) -> None:
        self.verbose = bool(verbose)
        self.dropped: dict[str, int] = {}

    def rules(self) -> Sequence[Rule]:
        return ()

    def check(self, sample: Any) -> CheckResult:
        for reason, fails in self.rules():
            if fails(sample):
                return CheckResult(False, reason)
        return CheckResult(True)

    def push(self, sample: Any) -> Iterable[Any]:
        verdict = self.check(sample)
        if verdict.is_valid:
            return (sample,)
        reason = verdict.reason or "unknown"
        self.dropped[reason] = self.dropped.get(reason, 0) + 1
        if self.verbose:
            simple_info(f"Data guard skip: reason={reason} sample={self._sample_info(sample)}", level="warning")
        return ()

    @staticmethod
    def _sample_info(sample: Any) -> Any:
        row = sample._raw if isinstance(sample, LLMSample) else sample
        if isinstance(row, dict):
            return {k: row[k] for k in _INFO_KEYS if k in row}
        text = repr(row)
        return text if len(text) <= 200 else text[:200] + "..."


class LLMRawRowGuard(LLMGuard):
    """Raw rows: must be dicts the schema handler accepts."""

    def __init__(self, assemble_context: Any = None, *, schema_handler: Optional[LLMSchemaHandler] = None,
                 verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.schema_handler = schema_handler or LLMPretrainTextSchemaHandler()

    def check(self, sample: Any) -> CheckResult:
        if not isinstance(sample, dict):
            return CheckResult(False, "raw.not_dict")
        reason = self.schema_handler.check_row(sample)  # the handler names its own reason
        return CheckResult(reason is None, reason)

    def fingerprint(self) -> str:
        return stable_fingerprint([type(self).__name__, repr(self.schema_handler)])


def _has_no_supervised_label(sample: LLMSample) -> bool:
    ignore = sample.tokenization_handler.ignore_index
    return all(lab == ignore for lab in sample.labels)


class LLMSampleGuard(LLMGuard):
    """Tokenised samples: non-empty, with at least one supervised label."""

    def rules(self) -> Sequence[Rule]:
        return (("sample.invalid_type", lambda s: not isinstance(s, LLMSample)),
                ("sample.empty_tokens", lambda s: s.tokenize().token_length <= 0),
                ("sample.no_supervised_tokens", _has_no_supervised_label))


def _bad_vector(key: str) -> Callable[[dict], bool]:
    def fails(item: dict) -> bool:
        v = item.get(key)
        return not (isinstance(v, torch.Tensor) and v.ndim == 1 and v.numel() > 0)

    return fails


def _shape_differs(key: str) -> Callable[[dict], bool]:
    return lambda item: item[key].shape != item["input_ids"].shape


class LLMModelInputGuard(LLMGuard):
    """Collated model inputs: 1-D non-empty aligned tensors, some supervised label, a positive sample count."""

    def __init__(self, assemble_context: Any = None, *, ignore_index: int = -100, verbose: bool = True) -> None:
        super().__init__(assemble_context, verbose=verbose)
        self.ignore_index = int(ignore_index)

    def rules(self) -> Sequence[Rule]:
        vectors = ("input_ids", "attention_mask", "labels", "pack_segment_ids")
        return (
            ("model_input.not_dict", lambda x: not isinstance(x, dict)),
            *((f"model_input.invalid_{k}", _bad_vector(k)) for k in vectors),
            ("model_input.attention_shape_mismatch", _shape_differs("attention_mask")),
            ("model_input.label_shape_mismatch", _shape_differs("labels")),
            ("model_input.pack_segment_shape_mismatch", _shape_differs("pack_segment_ids")),
            ("model_input.position_shape_mismatch",
             lambda x: "position_ids" in x and x["position_ids"].shape != x["input_ids"].shape),
            ("model_input.invalid_source_sample_num", lambda x: int(x.get("source_sample_num", 0)) <= 0),
            # labels are shifted by one in the loss, so the first position never counts
            ("model_input.no_supervised_tokens", lambda x: not bool(x["labels"][1:].ne(self.ignore_index).any())),
        )

    def fingerprint(self) -> str:
        return stable_fingerprint([type(self).__name__, self.ignore_index])
