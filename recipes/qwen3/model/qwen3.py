"""Qwen3 FLOPs accounting as a patchable method (reference: recipes/qwen3/model/qwen3.py:10-87)."""

from __future__ import annotations

from types import MethodType
from typing import Optional

import torch

from mvp_engine.models.qwen3 import qwen3_flops


def calculate_model_flops(self, *, batch_size: int, seq_len: int, attention_mask: Optional[torch.Tensor] = None,
                          is_training: bool = True, freeze_llm: bool = False,
                          attention_token_pairs: Optional[int] = None) -> float:
    """Per layer ``8BTH^2 + 4*pairs*H + 6BTHF`` plus ``2BTHV``; x3 for training."""
    if attention_token_pairs is not None:
        c = self.config
        B, T = int(batch_size), int(seq_len)
        H, F, V, L = c.hidden_size, c.intermediate_size, c.vocab_size, c.num_hidden_layers
        f = float(L * (8 * B * T * H * H + 4 * int(attention_token_pairs) * H + 6 * B * T * H * F) + 2 * B * T * H * V)
        return f if not is_training else f * (1.0 if freeze_llm else 3.0)
    return qwen3_flops(self.config, batch_size, seq_len, attention_mask, is_training, freeze_llm)


def patch_qwen3_model_flops(model):
    model.calculate_model_flops = MethodType(calculate_model_flops, model)
    return model
