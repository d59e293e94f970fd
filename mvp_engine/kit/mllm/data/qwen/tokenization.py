"""Import path of the Qwen-VL tokenisation handler (reference: mvp_engine/kit/mllm/data/qwen/tokenization.py).

The handler itself lives with the generic MLLM tokenisation code, beside the handler it specialises
(Qwen chat turns are closed by the chat template, so it appends no extra EOS)."""

from __future__ import annotations

from ..tokenization import QwenVLTokenizationHandler

__all__ = ["QwenVLTokenizationHandler"]
