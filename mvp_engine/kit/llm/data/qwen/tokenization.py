"""Qwen chat tokenisation: the chat template already closes turns, so no extra EOS."""

from dataclasses import dataclass

from ..tokenization import LLMTokenizationHandler


@dataclass(slots=True)
class QwenChatTokenizationHandler(LLMTokenizationHandler):
    add_eos: bool = False


__all__ = ["QwenChatTokenizationHandler"]
