"""Vision Transformer image classifier with Hugging Face ``ViTForImageClassification``
parameter names (reference model: recipes/vit_classification/model/vit.py:8-35).

Pre-LN encoder: patch embedding (a stride-P convolution, computed as one GEMM
over unfolded patches), a learned CLS token and position embeddings, L blocks
of ``x + Attn(LN(x))`` and ``x + MLP(LN(x))`` with exact GELU, a final
LayerNorm and a linear classifier on the CLS token.  Dropout probabilities are
honoured in training mode.

Precision: activations run in the parameters' dtype (bf16 under the native
data-parallel runtime, fp32 otherwise) with LayerNorm statistics and the
logits in fp32; an enclosing autocast region is switched off.  On CUDA the
projections run on the tcgen05 GEMM and attention on the varlen flash kernel
(one document per image, bidirectional, head_dim zero-padded to 128).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops.attention import attention_any_head_dim


@dataclass
class ViTConfig:
    image_size: int = 224
    patch_size: int = 16
    num_channels: int = 3
    hidden_size: int = 768
    intermediate_size: int = 3072
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    hidden_dropout_prob: float = 0.0
    attention_probs_dropout_prob: float = 0.0
    layer_norm_eps: float = 1e-12
    qkv_bias: bool = True
    num_labels: int = 1000
    initializer_range: float = 0.02
    model_type: str = "vit"

    def to_dict(self) -> dict:
        return asdict(self)


def _linear(x: torch.Tensor, lin: nn.Linear) -> torch.Tensor:
    if x.is_cuda and x.dtype == torch.bfloat16 and lin.weight.dtype == torch.bfloat16:
        y = ops.linear(x, lin.weight)
        return y if lin.bias is None else y + lin.bias
    return F.linear(x, lin.weight.to(x.dtype), None if lin.bias is None else lin.bias.to(x.dtype))


def _layer_norm(x: torch.Tensor, ln: nn.LayerNorm) -> torch.Tensor:
    """LayerNorm with fp32 statistics, result in the activation dtype."""
    return F.layer_norm(x.float(), ln.normalized_shape, ln.weight.float(), ln.bias.float(), ln.eps).to(x.dtype)


class ViTPatchEmbeddings(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.patch_size = c.patch_size
        self.num_patches = (c.image_size // c.patch_size) ** 2
        self.projection = nn.Conv2d(c.num_channels, c.hidden_size, kernel_size=c.patch_size, stride=c.patch_size)

    def forward(self, pixel_values: torch.Tensor) -> torch.Tensor:
        B, C, Hh, Ww = pixel_values.shape
        P = self.patch_size
        # unfold to [B, N, C*P*P] in (c, kh, kw) order == conv weight layout, then one GEMM
        patches = pixel_values.reshape(B, C, Hh // P, P, Ww // P, P).permute(0, 2, 4, 1, 3, 5)
        patches = patches.reshape(B, (Hh // P) * (Ww // P), C * P * P)
        w = self.projection.weight.reshape(self.projection.weight.shape[0], -1)
        if patches.is_cuda and patches.dtype == torch.bfloat16 and w.dtype == torch.bfloat16:
            return ops.linear(patches.contiguous(), w) + self.projection.bias
        return F.linear(patches, w.to(patches.dtype), self.projection.bias.to(patches.dtype))


class ViTEmbeddings(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.cls_token = nn.Parameter(torch.zeros(1, 1, c.hidden_size))
        self.patch_embeddings = ViTPatchEmbeddings(c)
        self.position_embeddings = nn.Parameter(torch.zeros(1, self.patch_embeddings.num_patches + 1, c.hidden_size))
        self.dropout = nn.Dropout(c.hidden_dropout_prob)

    def forward(self, pixel_values: torch.Tensor) -> torch.Tensor:
        x = self.patch_embeddings(pixel_values)
        cls = self.cls_token.to(x.dtype).expand(x.shape[0], -1, -1)
        x = torch.cat([cls, x], dim=1) + self.position_embeddings.to(x.dtype)
        return self.dropout(x)


class ViTSelfAttention(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.num_heads = c.num_attention_heads
        self.head_dim = c.hidden_size // c.num_attention_heads
        self.query = nn.Linear(c.hidden_size, c.hidden_size, bias=c.qkv_bias)
        self.key = nn.Linear(c.hidden_size, c.hidden_size, bias=c.qkv_bias)
        self.value = nn.Linear(c.hidden_size, c.hidden_size, bias=c.qkv_bias)
        self.dropout_p = c.attention_probs_dropout_prob


class ViTSelfOutput(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.dense = nn.Linear(c.hidden_size, c.hidden_size)
        self.dropout = nn.Dropout(c.hidden_dropout_prob)


class ViTAttention(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.attention = ViTSelfAttention(c)
        self.output = ViTSelfOutput(c)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        a = self.attention
        B, N, H = x.shape
        if x.is_cuda and x.dtype == torch.bfloat16 and not (self.training and a.dropout_p > 0):
            q, k, v = (_linear(x, lin).view(B * N, a.num_heads, a.head_dim) for lin in (a.query, a.key, a.value))
            cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device=x.device)
            o = attention_any_head_dim(q, k, v, cu, N, causal=False).reshape(B, N, H)
        else:
            q = _linear(x, a.query).view(B, N, a.num_heads, a.head_dim).transpose(1, 2)
            k = _linear(x, a.key).view(B, N, a.num_heads, a.head_dim).transpose(1, 2)
            v = _linear(x, a.value).view(B, N, a.num_heads, a.head_dim).transpose(1, 2)
            o = F.scaled_dot_product_attention(q, k, v, dropout_p=a.dropout_p if self.training else 0.0)
            o = o.transpose(1, 2).reshape(B, N, H)
        return self.output.dropout(_linear(o, self.output.dense))


class ViTIntermediate(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.dense = nn.Linear(c.hidden_size, c.intermediate_size)


class ViTOutput(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.dense = nn.Linear(c.intermediate_size, c.hidden_size)
        self.dropout = nn.Dropout(c.hidden_dropout_prob)


class ViTLayer(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.attention = ViTAttention(c)
        self.intermediate = ViTIntermediate(c)
        self.output = ViTOutput(c)
        self.layernorm_before = nn.LayerNorm(c.hidden_size, eps=c.layer_norm_eps)
        self.layernorm_after = nn.LayerNorm(c.hidden_size, eps=c.layer_norm_eps)

    @staticmethod
    def _ln(x: torch.Tensor, ln: nn.LayerNorm) -> torch.Tensor:
        return _layer_norm(x, ln)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attention(self._ln(x, self.layernorm_before))
        h = F.gelu(_linear(self._ln(x, self.layernorm_after), self.intermediate.dense))
        return x + self.output.dropout(_linear(h, self.output.dense))


class ViTEncoder(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.layer = nn.ModuleList([ViTLayer(c) for _ in range(c.num_hidden_layers)])


class ViTModel(nn.Module):
    def __init__(self, c: ViTConfig):
        super().__init__()
        self.config = c
        self.embeddings = ViTEmbeddings(c)
        self.encoder = ViTEncoder(c)
        self.layernorm = nn.LayerNorm(c.hidden_size, eps=c.layer_norm_eps)

    def forward(self, pixel_values: torch.Tensor) -> torch.Tensor:
        x = self.embeddings(pixel_values)
        for layer in self.encoder.layer:
            x = layer(x)
        return ViTLayer._ln(x, self.layernorm)


class ViTForImageClassification(nn.Module):
    _no_split_modules = ["ViTEmbeddings", "ViTLayer"]

    def __init__(self, config: ViTConfig):
        super().__init__()
        self.config = config
        self.num_labels = config.num_labels
        self.vit = ViTModel(config)
        self.classifier = nn.Linear(config.hidden_size, config.num_labels)

    @torch.no_grad()
    def init_param_(self, fqn: str, t: torch.Tensor, seed: Optional[int] = None) -> None:
        """HF ViT init: truncated-normal-free N(0, 0.02) weights, zero biases, unit LayerNorm."""
        if "layernorm" in fqn or fqn.endswith("layernorm.weight"):
            t.fill_(1.0 if fqn.endswith("weight") else 0.0)
            return
        if fqn.endswith("bias"):
            t.zero_()
            return
        import zlib

        g = torch.Generator(device=t.device)
        g.manual_seed((int(seed or 0) * 1_000_003 + zlib.crc32(fqn.encode())) % (1 << 62))
        t.copy_(torch.randn(t.shape, generator=g, device=t.device).mul_(self.config.initializer_range))

    @torch.no_grad()
    def init_weights(self, seed: Optional[int] = None) -> None:
        for name, p in self.named_parameters():
            buf = torch.empty(p.shape, dtype=torch.float32, device=p.device)
            self.init_param_(name, buf, seed)
            p.copy_(buf)

    def forward(self, pixel_values: torch.Tensor, labels: Optional[torch.Tensor] = None, **_: Any) -> dict:
        if pixel_values.is_cuda and torch.is_autocast_enabled("cuda"):
            with torch.autocast("cuda", enabled=False):
                return self.forward(pixel_values, labels)
        h = self.vit(pixel_values.to(self.classifier.weight.dtype))
        logits = F.linear(h[:, 0].float(), self.classifier.weight.float(), self.classifier.bias.float())
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits.float(), labels)
        return {"loss": loss, "logits": logits}


VIT_PRESETS = {
    "google/vit-base-patch16-224": dict(hidden_size=768, intermediate_size=3072, num_hidden_layers=12,
                                        num_attention_heads=12),
    "vit-tiny-patch16-224": dict(hidden_size=192, intermediate_size=768, num_hidden_layers=12,
                                 num_attention_heads=3),
}


def build_vit(name: str = "google/vit-base-patch16-224", *, seed: Optional[int] = 0, device: Any = None,
              **overrides: Any) -> ViTForImageClassification:
    cfg = ViTConfig(**{**VIT_PRESETS.get(name, {}), **overrides})
    with torch.device(device or "cpu"):
        model = ViTForImageClassification(cfg)
    model._init_seed = seed
    if device is None or torch.device(device).type != "meta":
        model.init_weights(seed)
    return model
