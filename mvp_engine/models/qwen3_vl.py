"""Qwen3-VL: vision tower + M-RoPE Qwen3 decoder, with Hugging Face parameter names
(``model.visual.*``, ``model.language_model.*``, ``lm_head``).

Reference behaviour mirrored (recipes/qwen3_vl/model/qwen3_vl.py:11-175 and the
HF modules the recipe loads):

* patch embedding: a Conv3d with kernel = stride = (2, 16, 16) over
  ``pixel_values [N, 3*2*16*16]``, computed as one linear layer in fp32
  (the reference swaps the conv for an fp32 ``F.linear``); on CUDA it runs as
  three bf16 tcgen05 GEMMs on a hi/lo split of both operands accumulated in
  fp32 (error ~2^-16 relative, same order as fp32 reduction error here);
* learned 48x48 position embeddings bilinearly interpolated to each image's
  patch grid, 2-D rotary embeddings (row, column) in the vision attention,
  bidirectional attention per image (``cu_seqlens`` from ``image_grid_thw``);
* pre-LN vision blocks (LayerNorm, qkv with bias, GELU-tanh MLP);
* 2x2 spatial merger to the LM width, and "deepstack" mergers whose outputs
  are added to the LM hidden states at image-token positions after the first
  decoder layers;
* the LM: Qwen3 decoder layers with interleaved multimodal RoPE (t/h/w
  sections [24, 20, 20]); chunked token cross-entropy on text labels.

Vision attention (head_dim 72) runs on the head_dim-128 tcgen05 kernel by
zero-padding q/k/v to 128 and passing the true softmax scale: padded lanes add
zero to every dot product and produce zero outputs, so the result is exact.
"""

from __future__ import annotations

import json
import math
import os
import zlib
from dataclasses import asdict, dataclass, field
from typing import Any, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops.attention import attention_any_head_dim, flash_attn_varlen
from .qwen3 import PackedContext, Qwen3Config, Qwen3DecoderLayer, Qwen3RMSNorm, _as_compute, shift_labels


@dataclass
class Qwen3VLVisionConfig:
    depth: int = 27
    hidden_size: int = 1152
    hidden_act: str = "gelu_pytorch_tanh"
    intermediate_size: int = 4304
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 16
    spatial_merge_size: int = 2
    temporal_patch_size: int = 2
    out_hidden_size: int = 4096
    num_position_embeddings: int = 2304
    deepstack_visual_indexes: list = field(default_factory=lambda: [8, 16, 24])
    initializer_range: float = 0.02


@dataclass
class Qwen3VLConfig:
    text_config: Qwen3Config = field(default_factory=lambda: Qwen3Config(rope_theta=5_000_000.0,
                                                                         max_position_embeddings=262144))
    vision_config: Qwen3VLVisionConfig = field(default_factory=Qwen3VLVisionConfig)
    mrope_section: list = field(default_factory=lambda: [24, 20, 20])
    image_token_id: int = 151655
    video_token_id: int = 151656
    vision_start_token_id: int = 151652
    vision_end_token_id: int = 151653
    tie_word_embeddings: bool = False
    model_type: str = "qwen3_vl"

    def to_dict(self) -> dict:
        return asdict(self)


QWEN3_VL_PRESETS = {
    "Qwen/Qwen3-VL-8B-Instruct": dict(),
    "Qwen/Qwen3-VL-2B-Instruct": dict(
        text=dict(hidden_size=2048, intermediate_size=6144, num_hidden_layers=28, num_attention_heads=16,
                  num_key_value_heads=8, tie_word_embeddings=True),
        vision=dict(depth=24, hidden_size=1024, intermediate_size=4096, num_heads=16, out_hidden_size=2048,
                    deepstack_visual_indexes=[5, 11, 17])),
    "mvp/qwen3-vl-tiny": dict(
        text=dict(vocab_size=151936, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=32768),
        vision=dict(depth=3, hidden_size=128, intermediate_size=256, num_heads=2, out_hidden_size=256,
                    deepstack_visual_indexes=[0, 1], num_position_embeddings=256)),
}


def load_qwen3_vl_config(name_or_path: str, **overrides: Any) -> Qwen3VLConfig:
    text: dict = {"rope_theta": 5_000_000.0, "max_position_embeddings": 262144}
    vision: dict = {}
    top: dict = {}
    cfg_file = os.path.join(name_or_path, "config.json")
    if os.path.isdir(name_or_path) and os.path.exists(cfg_file):
        with open(cfg_file) as f:
            d = json.load(f)
        text.update(d.get("text_config", {}))
        rp = text.get("rope_scaling") or text.get("rope_parameters") or {}
        if "mrope_section" in rp:
            top["mrope_section"] = rp["mrope_section"]
        vision.update(d.get("vision_config", {}))
        top.update({k: d[k] for k in ("image_token_id", "video_token_id", "vision_start_token_id",
                                      "vision_end_token_id", "tie_word_embeddings") if k in d})
    elif name_or_path in QWEN3_VL_PRESETS:
        p = QWEN3_VL_PRESETS[name_or_path]
        text.update(p.get("text", {}))
        vision.update(p.get("vision", {}))
    else:
        raise ValueError(f"Unknown Qwen3-VL model {name_or_path!r}")
    text.update(overrides.pop("text", {}))
    vision.update(overrides.pop("vision", {}))
    top.update(overrides)
    vfields = Qwen3VLVisionConfig.__dataclass_fields__
    return Qwen3VLConfig(text_config=Qwen3Config.from_dict(text),
                         vision_config=Qwen3VLVisionConfig(**{k: v for k, v in vision.items() if k in vfields}),
                         **{k: v for k, v in top.items() if k in Qwen3VLConfig.__dataclass_fields__})


# ------------------------------------------------------------------ helpers
def _linear(x: torch.Tensor, lin: nn.Linear) -> torch.Tensor:
    w = lin.weight
    if x.is_cuda and x.dtype == torch.bfloat16:
        y = ops.linear(x, _as_compute(w, x))
        return y if lin.bias is None else y + _as_compute(lin.bias, x)
    return F.linear(x, _as_compute(w, x), None if lin.bias is None else _as_compute(lin.bias, x))


def _ln(x: torch.Tensor, ln: nn.LayerNorm) -> torch.Tensor:
    """LayerNorm with bias: the sm_100a kernel pair on CUDA bf16, ``F.layer_norm`` elsewhere."""
    return ops.layer_norm(x, _as_compute(ln.weight, x), _as_compute(ln.bias, x), ln.eps)


def _linear_residual(x: torch.Tensor, lin: nn.Linear, residual: torch.Tensor) -> torch.Tensor:
    """``residual + (x @ W^T + b)``: GEMM without bias, then one fused bias + residual kernel on CUDA bf16."""
    if x.is_cuda and x.dtype == torch.bfloat16 and lin.bias is not None and residual.dtype == x.dtype:
        return ops.bias_residual(ops.linear(x, _as_compute(lin.weight, x)), _as_compute(lin.bias, x), residual)
    return residual + _linear(x, lin)


def _linear_gelu(x: torch.Tensor, lin: nn.Linear, approximate: str) -> torch.Tensor:
    """``gelu(x @ W^T + b)``: GEMM without bias, then one fused bias + GELU kernel on CUDA bf16."""
    if x.is_cuda and x.dtype == torch.bfloat16 and lin.bias is not None:
        return ops.bias_gelu(ops.linear(x, _as_compute(lin.weight, x)), _as_compute(lin.bias, x), approximate)
    return F.gelu(_linear(x, lin), approximate=approximate)


def linear_fp32_accurate(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor]) -> torch.Tensor:
    """x @ w.T + b in fp32 accuracy.  CUDA: hi/lo bf16 split, three tcgen05 GEMMs summed in fp32."""
    x = x.float()
    w = w.float()
    if not x.is_cuda:
        y = F.linear(x, w)
    else:
        return _SplitLinear.apply(x, w, b)
    return y if b is None else y + b.float()


class _SplitLinear(torch.autograd.Function):
    @staticmethod
    def _split(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        hi = t.to(torch.bfloat16)
        lo = (t - hi.float()).to(torch.bfloat16)
        return hi.contiguous(), lo.contiguous()

    @staticmethod
    def _product(ah, al, bh, bl, out, a_mn=False, b_mn=False):
        """out += (ah + al) (bh + bl)^T without the lo x lo term: three bf16 tcgen05 GEMMs accumulating in fp32
        (relative error ~2^-16, the fp32-accurate path at tensor-core speed)."""
        ops.gemm(al, bh, a_mn=a_mn, b_mn=b_mn, out=out, accumulate=True)
        ops.gemm(ah, bl, a_mn=a_mn, b_mn=b_mn, out=out, accumulate=True)
        ops.gemm(ah, bh, a_mn=a_mn, b_mn=b_mn, out=out, accumulate=True)

    @staticmethod
    def forward(ctx, x, w, b):
        xh, xl = _SplitLinear._split(x)
        wh, wl = _SplitLinear._split(w)
        out = torch.zeros(x.shape[0], w.shape[0], device=x.device, dtype=torch.float32)
        _SplitLinear._product(xh, xl, wh, wl, out)
        ctx.save_for_backward(x, w)
        ctx.has_b = b is not None
        ctx.acc = ops.grad_acc(w)
        return out if b is None else out + b.float()

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        g = g.float().contiguous()
        gh, gl = _SplitLinear._split(g)
        dx = dw = None
        if ctx.needs_input_grad[0]:  # dX = G W: W read N-major as the B operand
            dx = torch.zeros(g.shape[0], w.shape[1], device=g.device, dtype=torch.float32)
            wh, wl = _SplitLinear._split(w)
            _SplitLinear._product(gh, gl, wh, wl, dx, b_mn=True)
        if ctx.acc is not None or ctx.needs_input_grad[1]:  # dW = G^T X, added into the fp32 accumulator
            xh, xl = _SplitLinear._split(x)
            acc = ctx.acc if (ctx.acc is not None and ctx.acc.dtype == torch.float32 and ctx.acc.is_contiguous()
                              and ctx.acc.shape == w.shape) else None
            target = acc if acc is not None else torch.zeros_like(w, dtype=torch.float32)
            _SplitLinear._product(gh, gl, xh, xl, target, a_mn=True, b_mn=True)
            dw = None if acc is not None else target
        db = g.sum(0) if ctx.has_b and ctx.needs_input_grad[2] else None
        return dx, dw, db


# ---------------------------------------------------------------- vision tower
class Qwen3VLVisionPatchEmbed(nn.Module):
    def __init__(self, c: Qwen3VLVisionConfig):
        super().__init__()
        k = (c.temporal_patch_size, c.patch_size, c.patch_size)
        self.in_dim = c.in_channels * c.temporal_patch_size * c.patch_size * c.patch_size
        self.proj = nn.Conv3d(c.in_channels, c.hidden_size, kernel_size=k, stride=k, bias=True)

    def forward(self, pixel_values: torch.Tensor) -> torch.Tensor:
        w = self.proj.weight.reshape(self.proj.weight.shape[0], -1)
        return linear_fp32_accurate(pixel_values.reshape(-1, self.in_dim), w, self.proj.bias)


class Qwen3VLVisionMLP(nn.Module):
    def __init__(self, c: Qwen3VLVisionConfig):
        super().__init__()
        self.linear_fc1 = nn.Linear(c.hidden_size, c.intermediate_size, bias=True)
        self.linear_fc2 = nn.Linear(c.intermediate_size, c.hidden_size, bias=True)

    def forward(self, x, residual: Optional[torch.Tensor] = None):
        """``fc2(gelu(fc1(x)))``; with ``residual``, returns ``residual + that`` (bias and residual adds fused)."""
        h = _linear_gelu(x, self.linear_fc1, "tanh")
        if residual is not None:
            return _linear_residual(h, self.linear_fc2, residual)
        return _linear(h, self.linear_fc2)


class Qwen3VLVisionAttention(nn.Module):
    def __init__(self, c: Qwen3VLVisionConfig):
        super().__init__()
        self.num_heads = c.num_heads
        self.head_dim = c.hidden_size // c.num_heads
        self.qkv = nn.Linear(c.hidden_size, 3 * c.hidden_size, bias=True)
        self.proj = nn.Linear(c.hidden_size, c.hidden_size, bias=True)

    def forward(self, x: torch.Tensor, cu: torch.Tensor, max_len: int, cos: torch.Tensor, sin: torch.Tensor,
                residual: Optional[torch.Tensor] = None):
        """``cos`` / ``sin``: ``[N, head_dim / 2]`` fp32 of the rotary angles (both halves share them).

        With ``residual``, returns ``residual + attention output`` (bias and residual adds fused)."""
        N = x.shape[0]
        D = self.head_dim
        if x.is_cuda and x.dtype == torch.bfloat16 and D <= 128:
            # GEMM without bias; the RoPE kernel adds the qkv bias and writes q / k / v zero-padded to the
            # head_dim-128 attention layout directly
            qkv = ops.linear(x, _as_compute(self.qkv.weight, x))
            bias = _as_compute(self.qkv.bias, x) if self.qkv.bias is not None else None
            q, k, v = ops.vision_rope_pad(qkv, self.num_heads, cos, sin, 128, bias=bias)
            o = flash_attn_varlen(q, k, v, cu, max_len, causal=False, softmax_scale=D**-0.5)[..., :D]
            if residual is not None:
                return _linear_residual(o.reshape(N, -1), self.proj, residual)
            return _linear(o.reshape(N, -1), self.proj)
        qkv = _linear(x, self.qkv)
        q, k, v = qkv.view(N, 3, self.num_heads, D).unbind(1)
        c = torch.cat([cos, cos], -1).unsqueeze(1)
        s = torch.cat([sin, sin], -1).unsqueeze(1)
        qf, kf = q.float(), k.float()
        q = (qf * c + _rotate_half(qf) * s).to(x.dtype)
        k = (kf * c + _rotate_half(kf) * s).to(x.dtype)
        o = vision_attention(q, k, v, cu, max_len)
        out = _linear(o.reshape(N, -1), self.proj)
        return out if residual is None else residual + out


def _rotate_half(x):
    a, b = x.chunk(2, dim=-1)
    return torch.cat((-b, a), dim=-1)


def vision_attention(q, k, v, cu, max_len):
    """Bidirectional attention within each image; head_dim padded to 128 on CUDA (exact)."""
    return attention_any_head_dim(q, k, v, cu, max_len, causal=False)


class Qwen3VLVisionBlock(nn.Module):
    def __init__(self, c: Qwen3VLVisionConfig):
        super().__init__()
        self.norm1 = nn.LayerNorm(c.hidden_size, eps=1e-6)
        self.norm2 = nn.LayerNorm(c.hidden_size, eps=1e-6)
        self.attn = Qwen3VLVisionAttention(c)
        self.mlp = Qwen3VLVisionMLP(c)

    def forward(self, x, cu, max_len, cos, sin):
        x = self.attn(_ln(x, self.norm1), cu, max_len, cos, sin, residual=x)
        return self.mlp(_ln(x, self.norm2), residual=x)


class Qwen3VLVisionPatchMerger(nn.Module):
    def __init__(self, c: Qwen3VLVisionConfig, use_postshuffle_norm: bool = False):
        super().__init__()
        self.hidden_size = c.hidden_size * c.spatial_merge_size**2
        self.use_postshuffle_norm = use_postshuffle_norm
        self.norm = nn.LayerNorm(self.hidden_size if use_postshuffle_norm else c.hidden_size, eps=1e-6)
        self.linear_fc1 = nn.Linear(self.hidden_size, self.hidden_size)
        self.linear_fc2 = nn.Linear(self.hidden_size, c.out_hidden_size)

    def forward(self, x):
        x = _ln(x.reshape(-1, self.hidden_size), self.norm) if self.use_postshuffle_norm else \
            _ln(x, self.norm).reshape(-1, self.hidden_size)
        return _linear(_linear_gelu(x, self.linear_fc1, "none"), self.linear_fc2)


class Qwen3VLVisionModel(nn.Module):
    _no_split_modules = ["Qwen3VLVisionBlock"]

    def __init__(self, c: Qwen3VLVisionConfig):
        super().__init__()
        self.config = c
        self.patch_embed = Qwen3VLVisionPatchEmbed(c)
        self.pos_embed = nn.Embedding(c.num_position_embeddings, c.hidden_size)
        self.num_grid_per_side = int(c.num_position_embeddings**0.5)
        self.blocks = nn.ModuleList([Qwen3VLVisionBlock(c) for _ in range(c.depth)])
        self.merger = Qwen3VLVisionPatchMerger(c, use_postshuffle_norm=False)
        self.deepstack_visual_indexes = list(c.deepstack_visual_indexes)
        self.deepstack_merger_list = nn.ModuleList(
            [Qwen3VLVisionPatchMerger(c, use_postshuffle_norm=True) for _ in self.deepstack_visual_indexes])
        head_dim = c.hidden_size // c.num_heads
        self.rope_dim = head_dim // 2
        self.gradient_checkpointing = False

    def vision_metadata(self, grid_thw: torch.Tensor) -> dict[str, torch.Tensor]:
        """Host-side: rotary angles, interpolation indices/weights and cu_seqlens for the images."""
        return vision_metadata(grid_thw.tolist(), self.config, self.num_grid_per_side, self.rope_dim)

    def forward(self, pixel_values: torch.Tensor, grid_thw: torch.Tensor,
                meta: Optional[dict[str, torch.Tensor]] = None, dtype: torch.dtype = torch.float32):
        dev = pixel_values.device
        if meta is None:
            meta = self.vision_metadata(grid_thw.cpu())
        meta = {k: (v.to(dev, non_blocking=True) if isinstance(v, torch.Tensor) and k != "max_len" else v)
                for k, v in meta.items()}
        x = self.patch_embed(pixel_values)
        pe = self.pos_embed.weight
        pos = (F.embedding(meta["pos_idx"], _as_compute(pe, x)) * meta["pos_w"].unsqueeze(-1).to(x.dtype)).sum(0)
        x = (x + pos).to(dtype)
        ang = meta["rope_angles"]
        cos = ang.cos()
        sin = ang.sin()
        cu, max_len = meta["cu_seqlens"], int(meta["max_len"])
        deep = []
        for i, blk in enumerate(self.blocks):
            if self.gradient_checkpointing and self.training and torch.is_grad_enabled():
                from torch.utils.checkpoint import checkpoint

                x = checkpoint(blk, x, cu, max_len, cos, sin, use_reentrant=False)
            else:
                x = blk(x, cu, max_len, cos, sin)
            if i in self.deepstack_visual_indexes:
                deep.append(self.deepstack_merger_list[self.deepstack_visual_indexes.index(i)](x))
        return self.merger(x), deep


def vision_metadata(grid_thw: list, c: Qwen3VLVisionConfig, side: int, rope_dim: int) -> dict[str, torch.Tensor]:
    """Per-patch rotary angles (row/col), bilinear position-embedding taps and per-image cu_seqlens.

    Patches are ordered as the HF image processor emits them: for each image,
    2x2 merge blocks in raster order, the four patches of a block consecutive.
    """
    m = c.spatial_merge_size
    inv = 1.0 / (10000.0 ** (torch.arange(0, rope_dim, 2, dtype=torch.float32) / rope_dim))
    rows, cols, idx, wts, lens = [], [], [[], [], [], []], [[], [], [], []], []
    for t, h, w in grid_thw:
        t, h, w = int(t), int(h), int(w)
        br = torch.arange(h // m).view(-1, 1, 1, 1) * m + torch.arange(m).view(1, 1, -1, 1)
        bc = torch.arange(w // m).view(1, -1, 1, 1) * m + torch.arange(m).view(1, 1, 1, -1)
        r = br.expand(h // m, w // m, m, m).reshape(-1).repeat(t)
        cc = bc.expand(h // m, w // m, m, m).reshape(-1).repeat(t)
        rows.append(r)
        cols.append(cc)
        hi = torch.linspace(0, side - 1, h)
        wi = torch.linspace(0, side - 1, w)
        hf, wf = hi.int(), wi.int()
        hc, wc = (hf + 1).clamp(max=side - 1), (wf + 1).clamp(max=side - 1)
        dh, dw = hi - hf, wi - wf
        taps = [(hf, wf, (1 - dh)[:, None] * (1 - dw)[None]), (hf, wc, (1 - dh)[:, None] * dw[None]),
                (hc, wf, dh[:, None] * (1 - dw)[None]), (hc, wc, dh[:, None] * dw[None])]
        for j, (hh, ww, wt) in enumerate(taps):
            ii = (hh[:, None] * side + ww[None]).reshape(h // m, m, w // m, m).permute(0, 2, 1, 3).reshape(-1)
            wt = wt.reshape(h // m, m, w // m, m).permute(0, 2, 1, 3).reshape(-1)
            idx[j].append(ii.repeat(t))
            wts[j].append(wt.repeat(t))
        lens += [h * w] * t
    r = torch.cat(rows).float()
    cc = torch.cat(cols).float()
    angles = torch.cat([torch.outer(r, inv), torch.outer(cc, inv)], dim=-1)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    return {"rope_angles": angles, "pos_idx": torch.stack([torch.cat(i) for i in idx]).long(),
            "pos_w": torch.stack([torch.cat(w) for w in wts]), "cu_seqlens": cu,
            "max_len": torch.tensor(max(lens) if lens else 0)}


# ------------------------------------------------------------------ language model
class Qwen3VLTextModel(nn.Module):
    def __init__(self, c: Qwen3Config, mrope_section: list):
        super().__init__()
        self.config = c
        self.embed_tokens = nn.Embedding(c.vocab_size, c.hidden_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(c, i) for i in range(c.num_hidden_layers)])
        self.norm = Qwen3RMSNorm(c.hidden_size, c.rms_norm_eps)
        self.rope = ops.RopeCache(c.head_dim, c.rope_theta, mrope_section=mrope_section,
                                  max_positions=min(c.max_position_embeddings, 65536))
        self.gradient_checkpointing = False
        self.checkpoint_layers: Optional[int] = None


class Qwen3VLModel(nn.Module):
    def __init__(self, c: Qwen3VLConfig):
        super().__init__()
        self.visual = Qwen3VLVisionModel(c.vision_config)
        self.language_model = Qwen3VLTextModel(c.text_config, c.mrope_section)


class Qwen3VLForConditionalGeneration(nn.Module):
    _no_split_modules = ["Qwen3VLTextDecoderLayer", "Qwen3DecoderLayer", "Qwen3VLVisionBlock"]

    def __init__(self, config: Qwen3VLConfig):
        super().__init__()
        self.config = config
        self.model = Qwen3VLModel(config)
        tc = config.text_config
        self.lm_head = nn.Linear(tc.hidden_size, tc.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.language_model.embed_tokens.weight
        self.loss_chunk_size = 4096

    @property
    def visual(self):
        return self.model.visual

    def gradient_checkpointing_enable(self, gradient_checkpointing_kwargs: Optional[dict] = None) -> None:
        kw = gradient_checkpointing_kwargs or {}
        lm = self.model.language_model
        lm.gradient_checkpointing = True
        lm.checkpoint_layers = kw.get("num_layers")
        self.model.visual.gradient_checkpointing = True

    @torch.no_grad()
    def init_param_(self, fqn: str, t: torch.Tensor, seed: Optional[int] = None) -> None:
        last = fqn.rsplit(".", 1)[-1]
        parent = fqn.rsplit(".", 2)[-2] if fqn.count(".") >= 1 else ""
        if fqn.endswith("layernorm.weight") or fqn.endswith("_norm.weight") or fqn.endswith("model.norm.weight") \
                or (parent.startswith("norm") and last == "weight"):
            t.fill_(1.0)
            return
        if last == "bias":
            t.zero_()
            return
        g = torch.Generator(device=t.device)
        g.manual_seed((int(seed or 0) * 1_000_003 + zlib.crc32(fqn.encode())) % (1 << 62))
        t.copy_(torch.randn(t.shape, generator=g, device=t.device).mul_(0.02))

    @torch.no_grad()
    def init_weights(self, seed: Optional[int] = None) -> None:
        for name, p in self.named_parameters():
            buf = torch.empty(p.shape, dtype=torch.float32, device=p.device)
            self.init_param_(name, buf, seed)
            p.copy_(buf)

    def forward(self, input_ids: torch.Tensor, *args: Any, **kwargs: Any) -> dict:
        """The model manages its own precision (bf16 operands, fp32 accumulation and statistics);
        an enclosing CUDA autocast region would only re-cast what the kernels already decide."""
        if input_ids.is_cuda and torch.is_autocast_enabled("cuda"):
            with torch.autocast("cuda", enabled=False):
                return self._forward(input_ids, *args, **kwargs)
        return self._forward(input_ids, *args, **kwargs)

    def _forward(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None, cu_seq_lens_q: Optional[torch.Tensor] = None,
                max_length_q: Optional[int] = None, pixel_values: Optional[torch.Tensor] = None,
                image_grid_thw: Optional[torch.Tensor] = None, vision_meta: Optional[dict] = None,
                **unused: Any) -> dict:
        lm = self.model.language_model
        T = input_ids.numel()
        dev = input_ids.device
        dtype = torch.bfloat16 if input_ids.is_cuda else self.lm_head.weight.dtype
        ids = input_ids.reshape(-1)
        x = ops.embedding(ids, _as_compute(lm.embed_tokens.weight, torch.empty(0, dtype=dtype)),
                          getattr(lm, "_embed_anchor", None))
        image_mask = None
        deep: list = []
        if pixel_values is not None and image_grid_thw is not None and pixel_values.numel():
            img, deep = self.model.visual(pixel_values, image_grid_thw, vision_meta, dtype)
            image_mask = ids == self.config.image_token_id
            x = x.masked_scatter(image_mask.unsqueeze(-1), img.to(x.dtype))
        if cu_seq_lens_q is None:
            cu_seq_lens_q = torch.tensor([0, T], dtype=torch.int32, device=dev)
            max_length_q = T
        if position_ids is None:
            position_ids = torch.arange(T, device=dev).view(1, 1, T).expand(3, 1, T)
        pos = position_ids.reshape(position_ids.shape[0], -1) if position_ids.dim() == 3 else \
            position_ids.reshape(1, -1).expand(3, -1)
        ctx = PackedContext(pos, cu_seq_lens_q.to(dev, torch.int32), int(max_length_q or T), lm.rope)
        residual = None
        n_ckpt = len(lm.layers) if lm.checkpoint_layers is None else int(lm.checkpoint_layers)
        for i, layer in enumerate(lm.layers):
            if lm.gradient_checkpointing and self.training and i < n_ckpt and torch.is_grad_enabled():
                from torch.utils.checkpoint import checkpoint

                x, residual = checkpoint(layer, x, residual, ctx, use_reentrant=False)
            else:
                x, residual = layer(x, residual, ctx)
            if i < len(deep) and image_mask is not None:
                x = x.index_put((image_mask.nonzero().squeeze(1),), deep[i].to(x.dtype), accumulate=True)
        h, _ = lm.norm(x, residual)
        w = _as_compute(self.lm_head.weight, h)
        if labels is None:
            return {"logits": ops.linear(h, w).view(*input_ids.shape, -1)}
        return {"loss": ops.fused_linear_cross_entropy(h, w, shift_labels(labels).reshape(-1), self.loss_chunk_size),
                "logits": None}

    def calculate_model_flops(self, *, batch_size: int, seq_len: int, attention_token_pairs: Optional[int] = None,
                              image_grid_thw: Optional[torch.Tensor] = None, is_training: bool = True,
                              freeze_llm: bool = False, freeze_vit: bool = False, freeze_projector: bool = False,
                              **unused: Any) -> float:
        """MFU accounting of the reference (recipes/qwen3_vl/model/qwen3_vl.py:43-148), kept identical so MFU
        figures compare: LM as for Qwen3; ViT ``patch + L*(8 H^2 N + 4 H sum(N_i^2) + 4 H F N)``; merger
        ``2 N_merged (H m^2) H_out``.  Training multiplies by 3 for trained parts, 2 for a frozen part that
        still back-propagates to a trained part upstream of it, 1 otherwise."""
        tc, vc = self.config.text_config, self.config.vision_config
        pairs = attention_token_pairs if attention_token_pairs is not None else batch_size * seq_len * seq_len
        B, T = int(batch_size), int(seq_len)
        H, Fh, V, L = tc.hidden_size, tc.intermediate_size, tc.vocab_size, tc.num_hidden_layers
        lm = float(L * (8 * B * T * H * H + 4 * int(pairs) * H + 6 * B * T * H * Fh) + 2 * B * T * H * V)
        vit = merger = 0.0
        if image_grid_thw is not None and len(image_grid_thw):
            g = image_grid_thw.detach().to("cpu", torch.long).reshape(-1, 3)
            m = vc.spatial_merge_size
            n_i = (g[:, 0] * g[:, 1] * g[:, 2]).tolist()
            n_merged = int((g[:, 0] * (g[:, 1] // m) * (g[:, 2] // m)).sum())
            N = float(sum(n_i))
            Hv, Fv = vc.hidden_size, vc.intermediate_size
            patch = 2.0 * N * Hv * vc.in_channels * vc.temporal_patch_size * vc.patch_size ** 2
            vit = patch + vc.depth * (8 * Hv * Hv * N + 4 * Hv * float(sum(n * n for n in n_i)) + 4 * Hv * Fv * N)
            merger = 2.0 * n_merged * Hv * m * m * vc.out_hidden_size
        if not is_training:
            return lm + vit + merger
        llm_mult = 3.0 if not freeze_llm else (2.0 if (not freeze_projector or not freeze_vit) else 1.0)
        merger_mult = 3.0 if not freeze_projector else (2.0 if not freeze_vit else 1.0)
        vit_mult = 3.0 if not freeze_vit else 1.0
        return lm * llm_mult + merger * merger_mult + vit * vit_mult


def build_qwen3_vl(name_or_path: str = "Qwen/Qwen3-VL-8B-Instruct", *, seed: Optional[int] = 0,
                   dtype: torch.dtype = torch.float32, device: Any = None, **overrides: Any):
    cfg = load_qwen3_vl_config(name_or_path, **overrides)
    with torch.device(device or "cpu"):
        model = Qwen3VLForConditionalGeneration(cfg).to(dtype)
    model._init_seed = seed
    if device is None or torch.device(device).type != "meta":
        model.init_weights(seed)
    return model
