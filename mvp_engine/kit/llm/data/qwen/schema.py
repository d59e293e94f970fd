"""Qwen chat rows -> (prompt, response) segments (reference: mvp_engine/kit/llm/data/qwen/schema.py:27-179).

Each user/assistant pair becomes an unsupervised prompt segment and a
supervised response segment.  The split point is found by rendering the
conversation with and without the assistant turn through the tokenizer's chat
template (``apply_chat_template``); a tokenizer without one falls back to the
ChatML layout Qwen uses (``<|im_start|>role\\n...<|im_end|>\\n``).
``thinking_mode`` controls the ``<think>...</think>`` block: True keeps or
inserts an empty one, False strips it, "non-empty" strips only empty ones,
None leaves the text alone.  An inserted empty block counts as prompt text.
"""

from __future__ import annotations

import re
from collections.abc import Mapping
from typing import Any, Literal

from ..schema import LLMSchemaHandler
from ..types import LLMSegment

THOUGHT_PREFIX = "<think>\n"
THOUGHT_SUFFIX = "\n</think>\n\n"
THOUGHT_MARKERS = ("<think>", "</think>")
THOUGHT_PATTERN = re.compile(r"<think>(.*?)</think>\s*", re.DOTALL)
ROLE_MAP = {"system": "system", "user": "user", "human": "user", "assistant": "assistant", "gpt": "assistant",
            "model": "assistant"}


def _text(content: Any) -> str:
    if isinstance(content, str):
        return content
    if isinstance(content, list):
        parts = []
        for item in content:
            if isinstance(item, str):
                parts.append(item)
            elif isinstance(item, dict) and item.get("type", "text") == "text":
                parts.append(str(item.get("text", "")))
        return "".join(parts)
    raise ValueError("message content must be text")


def chatml(messages: list[dict[str, Any]], add_generation_prompt: bool) -> str:
    out = "".join(f"<|im_start|>{m['role']}\n{m['content']}<|im_end|>\n" for m in messages)
    return out + ("<|im_start|>assistant\n" if add_generation_prompt else "")


class QwenChatSchemaHandler(LLMSchemaHandler):
    def __init__(self, tokenizer: Any, *, thinking_mode: bool | None | Literal["non-empty"] = True) -> None:
        if thinking_mode not in (True, False, None, "non-empty"):
            raise ValueError("thinking_mode must be True, False, None, or 'non-empty'.")
        self.tokenizer = tokenizer
        self.thinking_mode = thinking_mode

    def _render(self, messages: list[dict[str, Any]], add_generation_prompt: bool) -> str:
        fn = getattr(self.tokenizer, "apply_chat_template", None)
        if callable(fn) and getattr(self.tokenizer, "chat_template", None):
            return fn(messages, tokenize=False, add_generation_prompt=add_generation_prompt)
        return chatml(messages, add_generation_prompt)

    def check_row(self, row: Mapping[str, Any]) -> str | None:
        msgs = row.get("messages") or row.get("conversations")
        if not isinstance(msgs, list) or not msgs:
            return "raw.invalid_messages"
        for m in msgs:
            if not isinstance(m, dict):
                return "raw.invalid_message"
            c = m.get("content", m.get("value"))
            if not isinstance(c, (str, list)):
                return "raw.invalid_message_content"
        return None

    @staticmethod
    def _normalize_message(m: dict[str, Any]) -> dict[str, str]:
        role = m.get("role") or m.get("from")
        norm = ROLE_MAP.get(role) if isinstance(role, str) else None
        if norm is None:
            raise ValueError(f"contains an invalid role: {role!r}")
        return {"role": norm, "content": _text(m.get("content", m.get("value")))}

    def _thinking(self, content: str) -> tuple[str, bool]:
        match = THOUGHT_PATTERN.search(content)
        empty = match is None or not match.group(1).strip()
        text = content
        if self.thinking_mode is False or (self.thinking_mode == "non-empty" and empty):
            text = THOUGHT_PATTERN.sub("", content).lstrip("\n")
        if all(mk in text for mk in THOUGHT_MARKERS) or self.thinking_mode is None:
            return text, False
        skip = self.thinking_mode is False or (self.thinking_mode == "non-empty" and empty)
        return f"{THOUGHT_PREFIX}{THOUGHT_SUFFIX}{text}", skip

    def normalize(self, row: Mapping[str, Any]) -> tuple[list[LLMSegment], dict[str, Any]]:
        reason = self.check_row(row)
        if reason is not None:
            raise ValueError(reason)
        msgs: list[tuple[dict[str, str], bool]] = []
        for raw in row.get("messages") or row.get("conversations"):
            m = self._normalize_message(raw)
            skip = False
            if m["role"] == "assistant":
                m["content"], skip = self._thinking(m["content"])
            msgs.append((m, skip))
        i = 0
        system: list[dict[str, str]] = []
        while i < len(msgs) and msgs[i][0]["role"] == "system":
            system.append(msgs[i][0])
            i += 1
        empty = f"{THOUGHT_PREFIX}{THOUGHT_SUFFIX}"
        segs: list[LLMSegment] = []
        while i + 1 < len(msgs):
            user, (asst, skip) = msgs[i][0], msgs[i + 1]
            if user["role"] != "user" or asst["role"] != "assistant":
                raise ValueError("conversation must contain user/assistant turn pairs after optional system messages.")
            src = self._render(system + [user], True)
            full = self._render(system + [user, asst], False)
            if not full.startswith(src):
                raise ValueError("tokenizer chat template does not preserve source prefix for target split.")
            tgt = full[len(src):]
            if skip and tgt.startswith(empty):
                src, tgt = src + empty, tgt[len(empty):]
            segs += [LLMSegment("text", False, src), LLMSegment("text", True, tgt)]
            system = []
            i += 2
        return [s for s in segs if s.value], {"schema": "qwen_chat"}
