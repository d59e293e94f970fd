"""Magic Transformer (reference: recipes/magic_transformer/model/source_model.py:14-585 with the
recipe's attention fix, recipes/magic_transformer/model/magic_transformer.py:16-78).

A research toy whose graph stresses data-parallel / sharding runtimes:

* two residual streams (``x_c`` content, ``x_m`` meta = ``meta_proj(embed)``);
* even layers send ``x_c`` through attention and ``x_m`` through the FFN, odd layers swap them;
* Mixture-of-Depths: a per-layer linear router scores tokens, only the top ``ratio * T`` tokens
  (kept in sequence order) enter attention / FFN, the rest skip the sub-layer;
* cross-layer KV reuse: an odd layer attends with the *un-rotated* K and V its preceding even layer
  projected (RoPE is applied once, at use);
* post-norms after each residual add, then a sigmoid fusion gate that mixes the two streams;
* router feedback: each layer keeps an EMA of its mean router score (a buffer, no gradient) and the
  next layer multiplies its pre-norm outputs by it;
* final norms, ``out_fusion`` over the concatenated streams, LM head tied to the embedding.

Routed tokens take rotary positions ``0..k-1`` of the compacted sequence by default
(``routed_positions="compacted"``, the behaviour of the reference); ``"original"`` rotates each
routed token by its position in the full sequence.  Parameter names follow the reference so
checkpoints interchange.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class TransformerConfig:
    vocab_size: int = 32000
    max_seq_len: int = 2048
    d_model: int = 512
    n_heads: int = 8
    n_kv_heads: int = 2
    n_layers: int = 8
    dropout: float = 0.1
    rope_base: float = 10000.0
    mod_top_k_ratio: float = 0.5
    dual_stream: bool = True
    router_ema_decay: float = 0.9
    routed_positions: str = "compacted"

    def __post_init__(self) -> None:
        if self.d_model % self.n_heads or self.n_heads % self.n_kv_heads:
            raise ValueError("d_model must divide by n_heads and n_heads by n_kv_heads")
        if self.n_layers % 2:
            raise ValueError("n_layers must be even (layers alternate in pairs)")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def ffn_hidden(self) -> int:
        return (int(8 * self.d_model / 3) + 63) // 64 * 64


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor, scale: Optional[torch.Tensor] = None) -> torch.Tensor:
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight
        return y if scale is None else y * scale


def rope_tables(positions: torch.Tensor, head_dim: int, base: float) -> tuple[torch.Tensor, torch.Tensor]:
    half = head_dim // 2
    inv = base ** (-torch.arange(half, device=positions.device, dtype=torch.float32) / half)
    ang = positions.float().unsqueeze(-1) * inv
    return ang.cos(), ang.sin()


def rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotary embedding of ``x [B, H, T, D]`` with tables ``[T, D/2]`` or ``[B, T, D/2]``."""
    a, b = x.chunk(2, dim=-1)
    if cos.dim() == 3:
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return torch.cat([a * cos - b * sin, a * sin + b * cos], dim=-1)


class GQAttention(nn.Module):
    def __init__(self, cfg: TransformerConfig) -> None:
        super().__init__()
        self.n_heads, self.n_kv_heads, self.head_dim = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        self.q_proj = nn.Linear(cfg.d_model, cfg.n_heads * cfg.head_dim, bias=False)
        self.k_proj = nn.Linear(cfg.d_model, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.v_proj = nn.Linear(cfg.d_model, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.out_proj = nn.Linear(cfg.n_heads * cfg.head_dim, cfg.d_model, bias=False)
        self.drop = nn.Dropout(cfg.dropout)

    def forward(self, x, cos, sin, mask=None, ext_kv=None):
        """GQA, causal unless ``mask`` (boolean keep-mask or additive float mask, broadcastable to
        ``[B, H, T, T]``) is given; returns ``(out, (k_unrotated, v))`` for reuse by the next layer."""
        B, T, _ = x.shape
        q = self.q_proj(x).view(B, T, self.n_heads, self.head_dim).transpose(1, 2)
        if ext_kv is None:
            k = self.k_proj(x).view(B, T, self.n_kv_heads, self.head_dim).transpose(1, 2)
            v = self.v_proj(x).view(B, T, self.n_kv_heads, self.head_dim).transpose(1, 2)
        else:
            k, v = ext_kv
        rep = self.n_heads // self.n_kv_heads
        kr = rotate(k, cos, sin).repeat_interleave(rep, dim=1)
        vr = v.repeat_interleave(rep, dim=1)
        o = F.scaled_dot_product_attention(rotate(q, cos, sin), kr, vr, attn_mask=mask, is_causal=mask is None,
                                           dropout_p=self.drop.p if self.training else 0.0)
        return self.out_proj(o.transpose(1, 2).reshape(B, T, -1)), (k, v)


class SwiGLUFFN(nn.Module):
    def __init__(self, cfg: TransformerConfig) -> None:
        super().__init__()
        h = cfg.ffn_hidden
        self.gate_proj = nn.Linear(cfg.d_model, h, bias=False)
        self.up_proj = nn.Linear(cfg.d_model, h, bias=False)
        self.down_proj = nn.Linear(h, cfg.d_model, bias=False)
        self.drop = nn.Dropout(cfg.dropout)

    def forward(self, x):
        return self.down_proj(self.drop(F.silu(self.gate_proj(x)) * self.up_proj(x)))


class MoDRouter(nn.Module):
    """Top-k token routing; returns (selected tokens, their indices in sequence order, router score)."""

    def __init__(self, cfg: TransformerConfig) -> None:
        super().__init__()
        self.ratio = cfg.mod_top_k_ratio
        self.router_linear = nn.Linear(cfg.d_model, 1, bias=False)

    def forward(self, x):
        B, T, D = x.shape
        k = max(1, int(T * self.ratio))
        score = self.router_linear(x)  # [B, T, 1]
        top = score.squeeze(-1).topk(k, dim=1, sorted=False).indices.sort(dim=1).values
        sel = torch.gather(x, 1, top.unsqueeze(-1).expand(-1, -1, D))
        return sel, top, score


def merge_routed(sel_out, x, top):
    """``x`` with the routed positions replaced by the sub-layer output: tokens the router skipped
    pass their (normalised) input through.  Out-of-place, so gradients stay dense."""
    return x.scatter(1, top.unsqueeze(-1).expand(-1, -1, x.shape[-1]), sel_out)


class DualStreamFusion(nn.Module):
    def __init__(self, d: int) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(2 * d, d, bias=False)

    def forward(self, xc, xm):
        g = torch.sigmoid(self.gate_proj(torch.cat([xc, xm], dim=-1)))
        return g * xc + (1 - g) * xm, (1 - g) * xc + g * xm


class TransformerBlock(nn.Module):
    def __init__(self, cfg: TransformerConfig, layer_idx: int) -> None:
        super().__init__()
        self.cfg, self.layer_idx, self.is_even = cfg, layer_idx, layer_idx % 2 == 0
        self.norm_c1, self.norm_m1 = RMSNorm(cfg.d_model), RMSNorm(cfg.d_model)
        self.norm_c2, self.norm_m2 = RMSNorm(cfg.d_model), RMSNorm(cfg.d_model)
        self.attn = GQAttention(cfg)
        self.ffn = SwiGLUFFN(cfg)
        self.router = MoDRouter(cfg)
        if cfg.dual_stream:
            self.fusion = DualStreamFusion(cfg.d_model)
        self.register_buffer("ema_score", torch.zeros(1))

    def _attend(self, x, rope, ext_kv):
        sel, top, score = self.router(x)
        k = sel.shape[1]
        if self.cfg.routed_positions == "original":
            cos, sin = rope_tables(top, self.cfg.head_dim, self.cfg.rope_base)
        else:
            cos, sin = rope[0][:k], rope[1][:k]
        out, kv = self.attn(sel, cos, sin, ext_kv=ext_kv)
        if self.training:
            with torch.no_grad():
                d = self.cfg.router_ema_decay
                self.ema_score.mul_(d).add_(score.detach().mean() * (1 - d))
        return merge_routed(out, x, top), kv

    def _ffn(self, x):
        sel, top, _ = self.router(x)
        return merge_routed(self.ffn(sel), x, top)

    def forward(self, xc, xm, rope, ext_kv=None, inject_scale=None):
        nc = self.norm_c1(xc, inject_scale)
        nm = self.norm_m1(xm, inject_scale)
        if self.is_even:
            a, kv = self._attend(nc, rope, ext_kv)
            xc, xm = xc + a, xm + self._ffn(nm)
        else:
            a, kv = self._attend(nm, rope, ext_kv)
            xm, xc = xm + a, xc + self._ffn(nc)
        xc, xm = self.norm_c2(xc), self.norm_m2(xm)
        if self.cfg.dual_stream:
            xc, xm = self.fusion(xc, xm)
        return xc, xm, kv, self.ema_score.view(1, 1, 1).expand(xc.shape[0], xc.shape[1], 1).clone()


class MagicTransformer(nn.Module):
    _no_split_modules = ["TransformerBlock"]

    def __init__(self, cfg: TransformerConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.meta_proj = nn.Linear(cfg.d_model, cfg.d_model, bias=False)
        self.drop = nn.Dropout(cfg.dropout)
        self.layers = nn.ModuleList([TransformerBlock(cfg, i) for i in range(cfg.n_layers)])
        self.norm_c, self.norm_m = RMSNorm(cfg.d_model), RMSNorm(cfg.d_model)
        self.out_fusion = nn.Linear(2 * cfg.d_model, cfg.d_model, bias=False)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.embed.weight
        cos, sin = rope_tables(torch.arange(cfg.max_seq_len), cfg.head_dim, cfg.rope_base)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self) -> None:
        """N(0, 0.02) matrices; residual-output projections N(0, 0.02 / sqrt(2 L))."""
        small = 0.02 / math.sqrt(2 * self.cfg.n_layers)
        for name, p in self.named_parameters():
            if p.dim() >= 2:
                p.normal_(0.0, small if name.split(".")[-2] in ("out_proj", "down_proj", "out_fusion") else 0.02)

    def forward(self, input_ids: torch.Tensor, **unused) -> torch.Tensor:
        B, T = input_ids.shape
        if T > self.cfg.max_seq_len:
            raise ValueError(f"sequence length {T} exceeds max_seq_len {self.cfg.max_seq_len}")
        e = self.drop(self.embed(input_ids))
        xc, xm = e, self.meta_proj(e)
        rope = (self.rope_cos[:T], self.rope_sin[:T])
        kv_even, scale = None, None
        for i, layer in enumerate(self.layers):
            xc, xm, kv, scale = layer(xc, xm, rope, ext_kv=kv_even if i % 2 else None, inject_scale=scale)
            if i % 2 == 0:
                kv_even = kv
        x = self.out_fusion(torch.cat([self.norm_c(xc), self.norm_m(xm)], dim=-1))
        return self.lm_head(x)

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 64, temperature: float = 1.0,
                 top_k: Optional[int] = 50) -> torch.Tensor:
        """Top-k sampling by re-running the window (no KV cache: routing depends on the whole window)."""
        for _ in range(max_new_tokens):
            logits = self(input_ids[:, -self.cfg.max_seq_len:])[:, -1] / max(temperature, 1e-6)
            if top_k:
                kth = logits.topk(min(top_k, logits.shape[-1])).values[:, -1:]
                logits = logits.masked_fill(logits < kth, float("-inf"))
            input_ids = torch.cat([input_ids, torch.multinomial(logits.softmax(-1), 1)], dim=1)
        return input_ids


def build_magic_transformer_model(config) -> MagicTransformer:
    return MagicTransformer(TransformerConfig(**config.model_dump()))
