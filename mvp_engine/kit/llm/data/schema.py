"""Row -> segment normalisation (reference: mvp_engine/kit/llm/data/schema.py:12-44)."""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

from .types import LLMSegment


class LLMSchemaHandler:
    """Extension point: validate a raw row cheaply and turn it into ordered segments."""

    def check_row(self, row: Mapping[str, Any]) -> str | None:
        return None

    def normalize(self, row: Mapping[str, Any]) -> tuple[list[LLMSegment], dict[str, Any]]:
        raise NotImplementedError


@dataclass(frozen=True, slots=True)
class LLMPretrainTextSchemaHandler(LLMSchemaHandler):
    """One document stored as text in ``text_field``; all of it supervised by default."""

    text_field: str = "data"
    loss: bool = True

    def check_row(self, row: Mapping[str, Any]) -> str | None:
        text = row.get(self.text_field)
        return None if isinstance(text, str) and text.strip() else "raw.invalid_text"

    def normalize(self, row: Mapping[str, Any]) -> tuple[list[LLMSegment], dict[str, Any]]:
        reason = self.check_row(row)
        if reason is not None:
            raise ValueError(reason)
        return [LLMSegment("text", self.loss, row[self.text_field])], {"text_field": self.text_field}


@dataclass(frozen=True, slots=True)
class LLMTokenIdsSchemaHandler(LLMSchemaHandler):
    """One pre-tokenised document in ``ids_field`` (synthetic or offline-tokenised data)."""

    ids_field: str = "input_ids"
    loss: bool = True

    def check_row(self, row: Mapping[str, Any]) -> str | None:
        ids = row.get(self.ids_field)
        return None if isinstance(ids, (list, tuple)) and len(ids) > 0 else "raw.invalid_token_ids"

    def normalize(self, row: Mapping[str, Any]) -> tuple[list[LLMSegment], dict[str, Any]]:
        reason = self.check_row(row)
        if reason is not None:
            raise ValueError(reason)
        return [LLMSegment("tokens", self.loss, list(row[self.ids_field]))], {"ids_field": self.ids_field}
