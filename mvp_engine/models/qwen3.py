"""Qwen3 dense decoder (text), written for the engine's packed-varlen hot path.

Parameter names and shapes follow Hugging Face ``Qwen3ForCausalLM`` so HF
safetensors and configs interoperate (``model.layers.{i}.self_attn.q_proj.weight``
...).  The forward works on packed token streams: the batch is flattened to
``[T]`` tokens, documents are delimited by ``cu_seqlens`` and attention never
crosses a document boundary; no 4-D masks are built.

Per layer on CUDA the sequence is
  RMSNorm(+residual) -> QKV GEMM -> QK-norm+RoPE -> varlen flash attention
  -> o GEMM -> RMSNorm(+residual) -> gate/up GEMM -> SwiGLU -> down GEMM
with every step a native sm_100a kernel (``mvp_engine.ops``).  The q/k/v and
gate/up weights are used as single fused GEMM operands: when the data-parallel
wrapper lays the parameters out contiguously it publishes fused views
(``layer._fused``); otherwise they are concatenated on the fly.

Reference behaviour mirrored: HF Qwen3 modules as loaded by
mvp_engine/kit/llm/model.py:19-60, the chunked per-token CE patch of
mvp_engine/kit/loss/token_loss.py:215-311 (labels shifted with -100 padding),
and the FLOPs formula of recipes/qwen3/model/qwen3.py:10-87.
"""

from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, dataclass, field
from typing import Any, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from .. import ops
from ..ops.attention import flash_attn_varlen


@dataclass
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 4096
    intermediate_size: int = 12288
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = False
    initializer_range: float = 0.02
    model_type: str = "qwen3"
    architectures: list = field(default_factory=lambda: ["Qwen3ForCausalLM"])
    torch_dtype: str = "bfloat16"
    _attn_implementation: str = "mvp_flash_varlen"

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "Qwen3Config":
        known = {k: v for k, v in d.items() if k in cls.__dataclass_fields__}
        cfg = cls(**known)
        if "head_dim" not in d and "hidden_size" in d:
            cfg.head_dim = cfg.hidden_size // cfg.num_attention_heads
        return cfg


# Architecture presets (public HF configs), used when no local config.json exists.  Every Qwen3 size
# uses 128-dim heads, which for several sizes is not hidden_size / heads.
QWEN3_PRESETS: dict[str, dict] = {
    "Qwen/Qwen3-0.6B": dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28, num_attention_heads=16,
                            num_key_value_heads=8, head_dim=128, tie_word_embeddings=True, max_position_embeddings=40960),
    "Qwen/Qwen3-1.7B": dict(hidden_size=2048, intermediate_size=6144, num_hidden_layers=28, num_attention_heads=16,
                            num_key_value_heads=8, head_dim=128, tie_word_embeddings=True, max_position_embeddings=40960),
    "Qwen/Qwen3-4B": dict(hidden_size=2560, intermediate_size=9728, num_hidden_layers=36, num_attention_heads=32,
                          num_key_value_heads=8, head_dim=128, tie_word_embeddings=True, max_position_embeddings=40960),
    "Qwen/Qwen3-8B": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                          num_key_value_heads=8, head_dim=128, max_position_embeddings=40960),
    "Qwen/Qwen3-8B-Base": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                               num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=32768),
    "Qwen/Qwen3-14B": dict(hidden_size=5120, intermediate_size=17408, num_hidden_layers=40, num_attention_heads=40,
                           num_key_value_heads=8, head_dim=128, max_position_embeddings=40960),
    "Qwen/Qwen3-32B": dict(hidden_size=5120, intermediate_size=25600, num_hidden_layers=64, num_attention_heads=64,
                           num_key_value_heads=8, head_dim=128, max_position_embeddings=40960),
    # tiny configs for tests and smoke runs
    "mvp/qwen3-tiny": dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                           max_position_embeddings=4096),
}


def load_qwen3_config(name_or_path: str, **overrides: Any) -> Qwen3Config:
    """Resolve a config from ``<path>/config.json`` or the preset table."""
    cfg_file = os.path.join(name_or_path, "config.json") if os.path.isdir(name_or_path) else None
    if cfg_file and os.path.exists(cfg_file):
        with open(cfg_file) as f:
            d = json.load(f)
    elif name_or_path in QWEN3_PRESETS:
        d = dict(QWEN3_PRESETS[name_or_path])
    else:
        raise ValueError(f"Unknown Qwen3 model {name_or_path!r}: no config.json and no preset")
    d.update(overrides)
    return Qwen3Config.from_dict(d)


class Qwen3RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None):
        y, h = ops.rms_norm(x, _as_compute(self.weight, x), self.variance_epsilon, residual=residual)
        return y if residual is None else (y, h)


def _as_compute(w: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """Weights enter the kernels in the activation dtype (bf16 under mixed precision)."""
    return w if w.dtype == like.dtype else w.to(like.dtype)


class Qwen3Attention(nn.Module):
    def __init__(self, config: Qwen3Config, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.head_dim = config.head_dim
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        H, D = config.hidden_size, config.head_dim
        self.q_proj = nn.Linear(H, self.num_heads * D, bias=False)
        self.k_proj = nn.Linear(H, self.num_kv_heads * D, bias=False)
        self.v_proj = nn.Linear(H, self.num_kv_heads * D, bias=False)
        self.o_proj = nn.Linear(self.num_heads * D, H, bias=False)
        self.q_norm = Qwen3RMSNorm(D, config.rms_norm_eps)
        self.k_norm = Qwen3RMSNorm(D, config.rms_norm_eps)
        self.scaling = D**-0.5


class Qwen3MLP(nn.Module):
    def __init__(self, config: Qwen3Config):
        super().__init__()
        H, F_ = config.hidden_size, config.intermediate_size
        self.gate_proj = nn.Linear(H, F_, bias=False)
        self.up_proj = nn.Linear(H, F_, bias=False)
        self.down_proj = nn.Linear(F_, H, bias=False)


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, config: Qwen3Config, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.self_attn = Qwen3Attention(config, layer_idx)
        self.mlp = Qwen3MLP(config)
        self.input_layernorm = Qwen3RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = Qwen3RMSNorm(config.hidden_size, config.rms_norm_eps)
        # Set by the data-parallel wrapper when q/k/v and gate/up are contiguous
        # in its parameter buffer: {"qkv": [3-way rows, H], "gate_up": [2F, H]}.
        self._fused: Optional[dict[str, torch.Tensor]] = None

    def fused_weight(self, name: str, like: torch.Tensor) -> torch.Tensor:
        if self._fused is not None and name in self._fused:
            return self._fused[name]
        a, m = self.self_attn, self.mlp
        parts = (a.q_proj, a.k_proj, a.v_proj) if name == "qkv" else (m.gate_proj, m.up_proj)
        return torch.cat([_as_compute(p.weight, like) for p in parts], dim=0)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor], ctx: "PackedContext"):
        """One decoder layer on flat tokens ``x [T, H]``; returns ``(mlp_out, residual)``.

        The residual add of the previous layer is fused into this layer's
        input RMSNorm: ``h = x + residual``.
        """
        attn = self.self_attn
        tp = getattr(self, "_tp", None)  # tensor-parallel runtime (column / row-parallel shards)
        Hq, Hkv, D = attn.num_heads, attn.num_kv_heads, attn.head_dim
        cp = ctx.cp
        if tp is None and (cp is None or not cp.ulysses_fused(x, Hq, Hkv, D)):
            return self._forward_plain(x, residual, ctx)
        if residual is None:
            hn = self.input_layernorm(x)
            h = x
        else:
            hn, h = self.input_layernorm(x, residual)
        if tp is None and cp is not None and cp.ulysses_fused(hn, Hq, Hkv, D):
            # context parallel (Ulysses) with the all-to-alls fused into the producing kernels
            o = cp.ulysses_block(hn, self.fused_weight("qkv", hn), _as_compute(attn.q_norm.weight, hn),
                                 _as_compute(attn.k_norm.weight, hn), _as_compute(attn.o_proj.weight, hn), ctx,
                                 Hq, Hkv, D, attn.q_norm.variance_epsilon, attn.scaling)
            hn2, h2 = self.post_attention_layernorm(o, h)
            gu = ops.linear(hn2, self.fused_weight("gate_up", hn2))
            return ops.swiglu_linear(gu, _as_compute(self.mlp.down_proj.weight, gu)), h2
        qkv = (tp.column_linear(hn, self.fused_weight("qkv", hn)) if tp is not None
               else ops.linear(hn, self.fused_weight("qkv", hn)))
        wq, wk = _as_compute(attn.q_norm.weight, hn), _as_compute(attn.k_norm.weight, hn)
        if cp is None and ctx.causal:  # one autograd node: all of q/k/v's gradients land in one dqkv buffer
            o = ops.qk_norm_rope_attention(qkv, Hq, Hkv, wq, wk, ctx.position_ids, ctx.rope,
                                           attn.q_norm.variance_epsilon, ctx.cu_seqlens, ctx.max_seqlen,
                                           attn.scaling)
        else:
            q, k = ops.qk_norm_rope(qkv, Hq, Hkv, wq, wk, ctx.position_ids, ctx.rope, attn.q_norm.variance_epsilon)
            v = qkv[:, (Hq + Hkv) * D:].view(-1, Hkv, D)
            o = ctx.attention(q, k, v, attn.scaling)
        o = o.reshape(o.shape[0], Hq * D)
        wo = _as_compute(attn.o_proj.weight, hn)
        o = tp.row_linear(o, wo) if tp is not None else ops.linear(o, wo)
        hn2, h2 = self.post_attention_layernorm(o, h)
        wgu = self.fused_weight("gate_up", hn2)
        gu = tp.column_linear(hn2, wgu) if tp is not None else ops.linear(hn2, wgu)
        wd = _as_compute(self.mlp.down_proj.weight, gu)
        if tp is not None:
            out = tp.row_linear(ops.swiglu(gu), wd)
        else:  # the activation is recomputed in the backward instead of being kept
            out = ops.swiglu_linear(gu, wd)
        return out, h2


    def _forward_plain(self, x: torch.Tensor, residual: Optional[torch.Tensor], ctx: "PackedContext"):
        """Single-rank / data-parallel / ring-CP layer: each RMSNorm and the GEMM it feeds are one autograd
        node that keeps the residual sum, not the normalised rows (``ops.rms_norm_linear``)."""
        attn = self.self_attn
        Hq, Hkv, D = attn.num_heads, attn.num_kv_heads, attn.head_dim
        ln1, ln2 = self.input_layernorm, self.post_attention_layernorm
        qkv, h = ops.rms_norm_linear(x, _as_compute(ln1.weight, x), self.fused_weight("qkv", x),
                                     ln1.variance_epsilon, residual=residual)
        wq, wk = _as_compute(attn.q_norm.weight, x), _as_compute(attn.k_norm.weight, x)
        if ctx.cp is None and ctx.causal:  # one autograd node: all of q/k/v's gradients land in one dqkv buffer
            o = ops.qk_norm_rope_attention(qkv, Hq, Hkv, wq, wk, ctx.position_ids, ctx.rope,
                                           attn.q_norm.variance_epsilon, ctx.cu_seqlens, ctx.max_seqlen,
                                           attn.scaling)
        else:
            q, k = ops.qk_norm_rope(qkv, Hq, Hkv, wq, wk, ctx.position_ids, ctx.rope, attn.q_norm.variance_epsilon)
            v = qkv[:, (Hq + Hkv) * D:].view(-1, Hkv, D)
            o = ctx.attention(q, k, v, attn.scaling)
        o = ops.linear(o.reshape(o.shape[0], Hq * D), _as_compute(attn.o_proj.weight, x))
        gu, h2 = ops.rms_norm_linear(o, _as_compute(ln2.weight, o), self.fused_weight("gate_up", o),
                                     ln2.variance_epsilon, residual=h)
        # the SwiGLU activation is recomputed in the backward instead of being kept
        return ops.swiglu_linear(gu, _as_compute(self.mlp.down_proj.weight, gu)), h2


@dataclass
class PackedContext:
    """Per-micro-batch metadata shared by every layer."""

    position_ids: torch.Tensor  # [A, T] int (A = 1 text RoPE, 3 M-RoPE)
    cu_seqlens: torch.Tensor  # [n_docs + 1] int32 on device
    max_seqlen: int
    rope: ops.RopeCache
    cp: Any = None  # context-parallel runtime (ring / ulysses), or None
    causal: bool = True

    def attention(self, q, k, v, scale):
        if self.cp is not None:
            return self.cp.attention(q, k, v, self, scale)
        return flash_attn_varlen(q, k, v, self.cu_seqlens, self.max_seqlen, causal=self.causal, softmax_scale=scale)


class Qwen3Model(nn.Module):
    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(config, i) for i in range(config.num_hidden_layers)])
        self.norm = Qwen3RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.rope = ops.RopeCache(config.head_dim, config.rope_theta, max_positions=config.max_position_embeddings)
        self.gradient_checkpointing = False
        self.checkpoint_layers: Optional[int] = None  # None: all layers when enabled

    def embed(self, input_ids: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        w = _as_compute(self.embed_tokens.weight, torch.empty(0, dtype=dtype))
        anchor = getattr(self, "_embed_anchor", None)
        return ops.embedding(input_ids.reshape(-1), w, anchor)

    def run_layers(self, x: torch.Tensor, ctx: PackedContext) -> torch.Tensor:
        residual = None
        n_ckpt = len(self.layers) if self.checkpoint_layers is None else int(self.checkpoint_layers)
        for i, layer in enumerate(self.layers):
            if self.gradient_checkpointing and self.training and i < n_ckpt and torch.is_grad_enabled():
                x, residual = checkpoint(layer, x, residual, ctx, use_reentrant=False)
            else:
                x, residual = layer(x, residual, ctx)
        out, _ = self.norm(x, residual)
        return out

    def forward(self, input_ids: torch.Tensor, ctx: PackedContext, dtype: torch.dtype = torch.bfloat16):
        x = self.embed(input_ids, dtype)
        return self.run_layers(x, ctx)


def shift_labels(labels: torch.Tensor) -> torch.Tensor:
    """``F.pad(labels, (0, 1), -100)[..., 1:]``: token t predicts label t+1 (last -> ignored)."""
    return F.pad(labels, (0, 1), value=-100)[..., 1:]


_shift_labels = shift_labels


def cu_seqlens_from_segments(segment_ids: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Flat-token ``cu_seqlens`` from per-row segment ids (0 = padding, its own segment).

    Documents never span rows; each change of id (or row start) opens a new document.
    """
    seg = segment_ids.reshape(segment_ids.shape[0], -1) if segment_ids.dim() > 1 else segment_ids.reshape(1, -1)
    B, T = seg.shape
    flat = seg.reshape(-1)
    starts = torch.ones_like(flat, dtype=torch.bool)
    starts[1:] = flat[1:] != flat[:-1]
    starts[::T] = True
    idx = torch.nonzero(starts, as_tuple=False).reshape(-1)
    cu = torch.cat([idx, torch.tensor([flat.numel()], device=idx.device)]).to(torch.int32)
    lens = cu[1:] - cu[:-1]
    return cu, int(lens.max().item()) if lens.numel() else 0


def positions_from_cu_seqlens(cu: torch.Tensor, total: int) -> torch.Tensor:
    """Per-document positions 0..len-1 for a flat packed stream."""
    ar = torch.arange(total, device=cu.device)
    seg = torch.searchsorted(cu[1:].long(), ar, right=True)
    return ar - cu[seg].long()


class Qwen3ForCausalLM(nn.Module):
    """HF-compatible Qwen3 causal LM; ``forward`` returns per-token loss when labels are given."""

    _no_split_modules = ["Qwen3DecoderLayer"]
    supports_sequence_parallel = True  # the embedding / loss work on this tensor rank's token slice
    base_model_prefix = "model"

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.config = config
        self.model = Qwen3Model(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self.loss_chunk_size = 4096

    def gradient_checkpointing_enable(self, gradient_checkpointing_kwargs: Optional[dict] = None) -> None:
        """Recompute decoder layers in backward (all, or the first ``num_layers``)."""
        kw = gradient_checkpointing_kwargs or {}
        self.model.gradient_checkpointing = True
        self.model.checkpoint_layers = kw.get("num_layers")

    def gradient_checkpointing_disable(self) -> None:
        self.model.gradient_checkpointing = False

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def init_param_(self, fqn: str, t: torch.Tensor, seed: Optional[int] = None) -> None:
        """HF-style init of one parameter in place: ones for norms, N(0, initializer_range)
        otherwise; the stream is seeded per (seed, name) so sharded and unsharded builds agree."""
        if fqn.endswith("norm.weight") or "layernorm" in fqn:
            t.fill_(1.0)
            return
        gen = torch.Generator(device=t.device)
        gen.manual_seed(_param_seed(seed, fqn))
        t.copy_(torch.randn(t.shape, generator=gen, device=t.device, dtype=torch.float32)
                .mul_(self.config.initializer_range))

    @torch.no_grad()
    def init_weights(self, seed: Optional[int] = None) -> None:
        for name, p in self.named_parameters():
            buf = torch.empty(p.shape, dtype=torch.float32, device=p.device)
            self.init_param_(name, buf, seed)
            p.copy_(buf)

    # ----------------------------------------------------------------- inputs
    def packed_context(self, input_ids: torch.Tensor, position_ids: Optional[torch.Tensor] = None,
                       cu_seq_lens_q: Optional[torch.Tensor] = None, max_length_q: Optional[int] = None,
                       pack_segment_ids: Optional[torch.Tensor] = None, cp: Any = None) -> PackedContext:
        T = input_ids.numel()
        if cu_seq_lens_q is None:
            if pack_segment_ids is not None:
                cu_seq_lens_q, max_length_q = cu_seqlens_from_segments(pack_segment_ids)
            else:
                B = input_ids.shape[0] if input_ids.dim() > 1 else 1
                L = T // B
                cu_seq_lens_q = torch.arange(0, T + 1, L, device=input_ids.device, dtype=torch.int32)
                max_length_q = L
        cu = cu_seq_lens_q.to(device=input_ids.device, dtype=torch.int32)
        if max_length_q is None:
            max_length_q = int((cu[1:] - cu[:-1]).max().item())
        if position_ids is None:
            position_ids = positions_from_cu_seqlens(cu, T)
        pos = position_ids.reshape(-1, T) if position_ids.dim() <= 2 else position_ids.reshape(position_ids.shape[0], -1)
        if input_ids.is_cuda:  # RoPE tables cover every position of the longest document
            self.model.rope.tables(input_ids.device, int(max_length_q))
        return PackedContext(pos, cu, int(max_length_q), self.model.rope, cp=cp)

    def forward(self, input_ids: torch.Tensor, *args: Any, **kwargs: Any) -> dict:
        """The model manages its own precision (bf16 operands, fp32 accumulation and statistics);
        an enclosing CUDA autocast region would only re-cast what the kernels already decide."""
        if input_ids.is_cuda and torch.is_autocast_enabled("cuda"):
            with torch.autocast("cuda", enabled=False):
                return self._forward(input_ids, *args, **kwargs)
        return self._forward(input_ids, *args, **kwargs)

    def _forward(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None, cu_seq_lens_q: Optional[torch.Tensor] = None,
                max_length_q: Optional[int] = None, pack_segment_ids: Optional[torch.Tensor] = None,
                ctx: Optional[PackedContext] = None, shift_labels: Optional[torch.Tensor] = None,
                **unused: Any) -> dict:
        """``shift_labels`` (labels already shifted by one, e.g. by context-parallel sharding)
        replaces ``labels``; with a context-parallel runtime attached (``_mvp_cp``) the inputs are
        this rank's tokens while ``cu_seq_lens_q`` describes the whole row."""
        if ctx is None:
            ctx = self.packed_context(input_ids, position_ids, cu_seq_lens_q, max_length_q, pack_segment_ids,
                                      cp=getattr(self, "_mvp_cp", None))
        dtype = torch.bfloat16 if input_ids.is_cuda else self.lm_head.weight.dtype
        if torch.is_autocast_enabled() and not input_ids.is_cuda:
            dtype = torch.get_autocast_dtype("cpu")
        tp = getattr(self, "_mvp_tp", None)
        local = tp.seq_slice(input_ids.numel()) if tp is not None else slice(None)
        h = self.model(input_ids.reshape(-1)[local], ctx, dtype)  # sequence parallel: this rank's tokens
        w = _as_compute(self.lm_head.weight, h)
        if labels is None and shift_labels is None:
            if tp is not None and tp.sequence_parallel:
                raise NotImplementedError("logits under sequence parallelism: pass labels for the loss")
            return {"logits": ops.linear(h, w).view(*input_ids.shape, -1)}
        flat_labels = (shift_labels if shift_labels is not None else _shift_labels(labels)).reshape(-1)[local]
        # the training loop may promise the loss's per-token gradient (``loss_grad_hint``): the LM head then
        # finishes its backward inside the forward, without recomputing the logits (not under TP)
        hint = getattr(self, "loss_grad_hint", None) if tp is None else None
        loss = ops.fused_linear_cross_entropy(h, w, flat_labels, self.loss_chunk_size, grad_hint=hint)
        return {"loss": loss, "logits": None}

    # ------------------------------------------------------------------ flops
    def calculate_model_flops(self, *, batch_size: int, seq_len: int, attention_mask: Optional[torch.Tensor] = None,
                              is_training: bool = True, freeze_llm: bool = False) -> float:
        """Logical FLOPs with the reference's formula (recipes/qwen3/model/qwen3.py:10-47):
        per layer ``8BTH^2 + 4*pairs*H + 6BTHF``, plus ``2BTHV``; x3 when training."""
        return qwen3_flops(self.config, batch_size, seq_len, attention_mask, is_training, freeze_llm)


def _param_seed(seed: Optional[int], fqn: str) -> int:
    import zlib

    return (int(seed or 0) * 1_000_003 + zlib.crc32(fqn.encode())) % (1 << 62)


def attention_pairs(batch: int, tokens: int, attention_mask: Optional[torch.Tensor]) -> int:
    """Σ len² over documents (packed segment ids > 1) or valid lengths (0/1 masks)."""
    if attention_mask is None or attention_mask.dim() != 2:
        return batch * tokens * tokens
    m = attention_mask.detach().to("cpu", torch.long)
    if m.numel() and int(m.max()) > 1:
        total = 0
        for row in m:
            ids = row[row > 0]
            if ids.numel():
                total += int(torch.bincount(ids).pow(2).sum())
        return total
    lens = m.ne(0).sum(-1)
    return int(lens.pow(2).sum())


def qwen3_flops(config, batch_size, seq_len, attention_mask=None, is_training=True, freeze_llm=False) -> float:
    B, T = int(batch_size), int(seq_len)
    H, F_, V, L = config.hidden_size, config.intermediate_size, config.vocab_size, config.num_hidden_layers
    pairs = attention_pairs(B, T, attention_mask)
    per_layer = 8 * B * T * H * H + 4 * pairs * H + 6 * B * T * H * F_
    flops = float(L * per_layer + 2 * B * T * H * V)
    if not is_training:
        return flops
    return flops * (1.0 if freeze_llm else 3.0)


def build_qwen3(name_or_path: str = "Qwen/Qwen3-8B-Base", *, seed: Optional[int] = 0,
                device: Optional[torch.device] = None, dtype: torch.dtype = torch.float32,
                **overrides: Any) -> Qwen3ForCausalLM:
    """Random-init model from a preset or local config.json (meta-device friendly)."""
    cfg = load_qwen3_config(name_or_path, **overrides)
    with torch.device(device or "cpu"):
        model = Qwen3ForCausalLM(cfg).to(dtype)
    model._init_seed = seed
    if device is None or torch.device(device).type != "meta":
        model.init_weights(seed)
    return model
