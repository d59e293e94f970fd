"""The Magic Transformer's building blocks under the reference's module path
(recipes/magic_transformer/model/source_model.py), with its helper functions' signatures.

The blocks are this recipe's (``magic_transformer.py``, with its own constructor and forward arguments:
the fusion and block modules take the recipe config and one stream pair per call); the helpers below
adapt the reference's call forms onto them."""

from __future__ import annotations

import torch

from .magic_transformer import (DualStreamFusion, GQAttention, MagicTransformer, MoDRouter, RMSNorm, SwiGLUFFN,
                                TransformerBlock, TransformerConfig, rope_tables, rotate)


def build_rope_cache(seq_len: int, head_dim: int, base: float = 10000.0, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin tables ``[seq_len, head_dim / 2]`` for positions 0 .. seq_len-1."""
    return rope_tables(torch.arange(seq_len, device=device), head_dim, base)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotary embedding of ``x [B, H, T, D]`` with ``[T, D/2]`` tables."""
    return rotate(x, cos, sin)


def scatter_back(selected_out: torch.Tensor, rest_x: torch.Tensor, top_indices: torch.Tensor,
                 rest_indices: torch.Tensor, seq_len: int) -> torch.Tensor:
    """``[B, seq_len, D]`` with the routed tokens' outputs at ``top_indices`` and the skipped tokens at
    ``rest_indices`` (the two index sets partition the sequence)."""
    B, _, D = selected_out.shape
    out = selected_out.new_empty(B, seq_len, D)
    out = out.scatter(1, top_indices.unsqueeze(-1).expand(-1, -1, D), selected_out)
    return out.scatter(1, rest_indices.unsqueeze(-1).expand(-1, -1, D), rest_x.to(out.dtype))


__all__ = ["DualStreamFusion", "GQAttention", "MagicTransformer", "MoDRouter", "RMSNorm", "SwiGLUFFN",
           "TransformerBlock", "TransformerConfig", "apply_rope", "build_rope_cache", "scatter_back"]
