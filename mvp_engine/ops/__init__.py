"""Hot-path operators of the engine.

On CUDA every operator here runs a hand-written sm_100a kernel from
``mvp_engine._C`` (tcgen05 GEMM, fused norms, RoPE, SwiGLU, cross-entropy,
AdamW, embedding); a missing extension raises.  On CPU the same operators
run plain PyTorch math with identical semantics, which is what the CPU test
suite and the gloo multi-process tests exercise.

Weight gradients: a weight tensor may carry a ``_mvp_grad_acc`` attribute
(an fp32 tensor of the same shape, usually a view into a flat gradient
buffer owned by the data-parallel wrapper).  When present, the backward of
:func:`linear` / :func:`embedding` accumulates the weight gradient straight
into it with the GEMM's fp32 accumulate epilogue, and no per-parameter
gradient tensor is materialised.  The forward reads the attribute (``grad_acc``)
and keeps it on the autograd context: under activation checkpointing the
backward sees a detached alias of the weight, without the attribute.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn.functional as F

from . import _ext

__all__ = [
    "gemm",
    "linear",
    "rms_norm",
    "rms_norm_linear",
    "qk_norm_rope",
    "qk_norm_rope_attention",
    "RopeCache",
    "swiglu",
    "swiglu_linear",
    "embedding",
    "fused_linear_cross_entropy",
    "adamw_step_",
    "sumsq",
    "layer_norm",
    "bias_gelu",
    "vision_rope_pad",
    "bias_residual",
]


def _native(t: torch.Tensor) -> bool:
    if not t.is_cuda:
        return False
    if not _ext.native_required():
        return _ext.available()
    return True


# --------------------------------------------------------------------- GEMM
class GatherJob:
    """An FSDP shard gather waiting for a GEMM to carry it (see ``NativeFSDP``).

    The next large enough :func:`gemm` on the CUDA path launches the two-SM kernel with ``copy_ctas``
    extra CTAs that pull every rank's bf16 shard into ``slot``; ``consumed`` then becomes True.  The
    runtime that queued the job launches the stand-alone pull instead if no GEMM took it by the time
    the gathered weights are needed."""

    def __init__(self, peer_bufs: list[int], peer_flags: list[int], offset: int, shard: int, epoch: int,
                 slot: torch.Tensor, copy_ctas: int, min_mnk: int, timeout_s: float = 10.0) -> None:
        """``min_mnk``: smallest GEMM (in FLOPs, 2 M N K) that may carry the copy -- one that runs about as long
        as the copy, so the copy CTAs finish within the GEMM."""
        self.args = (list(peer_bufs), list(peer_flags), int(offset), int(shard), int(epoch))
        self.slot = slot
        self.copy_ctas = int(copy_ctas)
        self.min_mnk = int(min_mnk)
        self.timeout_ns = int(timeout_s * 1e9)
        self.consumed = False


_pending_gather: Optional[GatherJob] = None


def set_pending_gather(job: Optional[GatherJob]) -> None:
    global _pending_gather
    _pending_gather = job


def pending_gather() -> Optional[GatherJob]:
    return _pending_gather


def _carry_pending_gather(a, a_mn, b, b_mn, out, accumulate, M: int, N: int, K: int) -> bool:
    """Launch this GEMM with the pending gather's copy CTAs if it is large enough; True when launched."""
    global _pending_gather
    job = _pending_gather
    if job is None or M < 256 or N < 256 or 2 * M * N * K < job.min_mnk or a.dtype != torch.bfloat16:
        return False
    if os.environ.get("MVP_GEMM_PAIR", "1") == "0":  # the carrying kernel is the two-SM one
        return False
    _pending_gather = None
    bufs, flags, off, shard, epoch = job.args
    _ext.ext().gemm_pair_gather(a, a_mn, b, b_mn, out, accumulate, _ext.status_buffer(a.device).data_ptr(), bufs,
                                flags, off, shard, epoch, job.slot, job.copy_ctas, job.timeout_ns)
    job.consumed = True
    return True


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    out: Optional[torch.Tensor] = None,
    accumulate: bool = False,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """C (+)= A * B^T on the tcgen05 tensor core.

    ``a`` is ``[M, K]`` (or ``[K, M]`` when ``a_mn``), ``b`` is ``[N, K]`` (or
    ``[K, N]`` when ``b_mn``).  The result is ``[M, N]`` in ``out_dtype`` (bf16 or
    fp32); ``accumulate=True`` adds into an fp32 ``out``.
    """
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if not _native(a):
        A = a.t() if a_mn else a
        B = b if b_mn else b.t()
        res = A.float() @ B.float()
        if out is None:
            return res.to(out_dtype)
        if accumulate:
            out.add_(res)
        else:
            out.copy_(res)
        return out
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    K = a.shape[0] if a_mn else a.shape[1]
    if _pending_gather is not None and _carry_pending_gather(a, a_mn, b, b_mn, out, accumulate, M, N, K):
        return out
    _ext.ext().gemm(a, a_mn, b, b_mn, out, accumulate, _ext.status_buffer(a.device).data_ptr())
    return out


def grad_acc(w: torch.Tensor) -> Optional[torch.Tensor]:
    """The fp32 gradient accumulator attached to weight ``w`` (``None`` if it has none)."""
    return getattr(w, "_mvp_grad_acc", None)


def _wgrad(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor,
           acc: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """dW = dY^T X, accumulated into ``acc`` (default: ``w._mvp_grad_acc``) when present."""
    acc = acc if acc is not None else grad_acc(w)
    if acc is not None:
        gemm(dy2, x2, a_mn=True, b_mn=True, out=acc, accumulate=True)
        return None
    return gemm(dy2, x2, a_mn=True, b_mn=True, out_dtype=w.dtype if w.dtype != torch.float32 else torch.float32)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0:
            x2 = x2.contiguous()
        y = gemm(x2, w)
        ctx.save_for_backward(x2, w)
        ctx.acc = grad_acc(w)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dy2, w, b_mn=True).view(*dy.shape[:-1], w.shape[1])
        dw = None
        if ctx.acc is not None or ctx.needs_input_grad[1]:
            dw = _wgrad(dy2, x2, w, ctx.acc)
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` (no bias) on the tcgen05 GEMM; eager ``F.linear`` on CPU."""
    if not _native(x):
        return F.linear(x, w.to(x.dtype))
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    if w.dtype != torch.bfloat16:
        raise TypeError("linear: the CUDA path expects bf16 weights (cast by the data-parallel wrapper)")
    return _Linear.apply(x, w)


# ------------------------------------------------------------------ RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        r2 = residual.reshape(-1, shape[-1]).contiguous() if residual is not None else None
        outs = _ext.ext().rmsnorm_fwd(x2, r2, w, eps)
        y, rstd = outs[0], outs[1]
        h = outs[2] if residual is not None else x2
        ctx.save_for_backward(h, rstd, w)
        ctx.acc = grad_acc(w)
        ctx.has_res = residual is not None
        ctx.shape = shape
        return y.view(shape), h.view(shape)

    @staticmethod
    def backward(ctx, dy, dh):
        h, rstd, w = ctx.saved_tensors
        H = ctx.shape[-1]
        dy2 = dy.reshape(-1, H).contiguous()
        dh2 = dh.reshape(-1, H).contiguous() if dh is not None else None
        acc = ctx.acc if (ctx.acc is not None and ctx.acc.is_contiguous() and ctx.acc.dtype == torch.float32) else None
        outs = _ext.ext().rmsnorm_bwd(dy2, h, rstd, w, dh2, True, dw_acc=acc)
        dx = outs[0].view(ctx.shape)
        if acc is not None:  # added into the fp32 accumulator by the kernel
            dw = None
        elif ctx.acc is not None:
            ctx.acc.add_(outs[1])
            dw = None
        else:
            dw = outs[1].to(w.dtype)
        return dx, dw, (dx if ctx.has_res else None), None


class _NormLinear(torch.autograd.Function):
    """``(rmsnorm(x + residual) * w_norm) @ w_lin^T`` plus the sum ``h = x + residual``, keeping only
    ``h`` and the row scales for the backward.

    The normalised rows (the GEMM's input) are not held from forward to backward: the backward
    recomputes them from ``h`` in one bandwidth-bound pass before the weight-gradient GEMM.  Decoder
    layers use this for the input and post-attention norms; the activation memory saved lets more
    layers skip activation checkpointing."""

    @staticmethod
    def forward(ctx, x, residual, w_norm, w_lin, eps):
        shape = x.shape
        H = shape[-1]
        x2 = x.reshape(-1, H).contiguous()
        r2 = residual.reshape(-1, H).contiguous() if residual is not None else None
        ext = _ext.ext()
        outs = ext.rmsnorm_fwd(x2, r2, w_norm, eps)
        hn, rstd = outs[0], outs[1]
        h = outs[2] if residual is not None else x2
        y = gemm(hn, w_lin)
        ctx.save_for_backward(h, rstd, w_norm, w_lin)
        ctx.accs = (grad_acc(w_norm), grad_acc(w_lin))
        ctx.has_res = residual is not None
        ctx.shape = shape
        ctx.eps = eps
        return y.view(*shape[:-1], w_lin.shape[0]), h.view(shape)

    @staticmethod
    def backward(ctx, dy, dh):
        h, rstd, w_norm, w_lin = ctx.saved_tensors
        acc_n, acc_l = ctx.accs
        H = ctx.shape[-1]
        ext = _ext.ext()
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        hn = ext.rmsnorm_fwd(h, None, w_norm, ctx.eps)[0]  # the GEMM input, recomputed
        dw_lin = None
        if acc_l is not None or ctx.needs_input_grad[3]:
            dw_lin = _wgrad(dy2, hn, w_lin, acc_l)
        del hn
        dhn = gemm(dy2, w_lin, b_mn=True)
        dh2 = dh.reshape(-1, H).contiguous() if dh is not None else None
        acc = acc_n if (acc_n is not None and acc_n.is_contiguous() and acc_n.dtype == torch.float32) else None
        outs = ext.rmsnorm_bwd(dhn, h, rstd, w_norm, dh2, True, dw_acc=acc)
        dx = outs[0].view(ctx.shape)
        if acc is not None:
            dw_norm = None
        elif acc_n is not None:
            acc_n.add_(outs[1])
            dw_norm = None
        else:
            dw_norm = outs[1].to(w_norm.dtype)
        return dx, (dx if ctx.has_res else None), dw_norm, dw_lin, None


def rms_norm_linear(x: torch.Tensor, w_norm: torch.Tensor, w_lin: torch.Tensor, eps: float,
                    residual: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(linear(rmsnorm(h) * w_norm, w_lin), h)`` with ``h = x + residual`` (or ``x``), without keeping the
    normalised rows for the backward (see :class:`_NormLinear`)."""
    if not _native(x) or x.dtype != torch.bfloat16 or w_lin.dtype != torch.bfloat16:
        y, h = rms_norm(x, w_norm, eps, residual=residual)
        return linear(y, w_lin), h
    return _NormLinear.apply(x, residual, w_norm, w_lin, float(eps))


def _rms_norm_eager(x, w, eps):
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return w.to(x.dtype) * (xf * torch.rsqrt(var + eps)).to(x.dtype)


def rms_norm(
    x: torch.Tensor, w: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None
) -> tuple[torch.Tensor, torch.Tensor]:
    """Return ``(rmsnorm(h) * w, h)`` with ``h = x + residual`` (or ``x``)."""
    if not _native(x):
        h = x if residual is None else (x + residual)
        return _rms_norm_eager(h, w, eps), h
    return _RMSNorm.apply(x, w, residual, float(eps))


# ------------------------------------------------------------ QK-norm + RoPE
class RopeCache:
    """cos/sin tables for (M-)RoPE, built the way HF's rotary embedding builds them.

    ``inv_freq = 1 / theta^(arange(0, D, 2)/D)`` in fp32 and
    ``angle[p, i] = p * inv_freq[i]`` in fp32; the kernels round cos/sin to
    bf16 at use, as HF casts them to the activation dtype.  ``mrope_section``
    (Qwen3-VL, e.g. ``[24, 20, 20]``) assigns each frequency to the t/h/w
    position axis with the interleaved layout.
    """

    def __init__(
        self, head_dim: int, theta: float, mrope_section: Optional[list[int]] = None, max_positions: int = 32768
    ):
        self.head_dim = head_dim
        self.max_positions = int(max_positions)
        self.theta = float(theta)
        self.mrope_section = list(mrope_section) if mrope_section else None
        ar = torch.arange(0, head_dim, 2, dtype=torch.int64, device="cpu").float()
        self.inv_freq = 1.0 / (self.theta ** (ar / head_dim))
        axis = torch.zeros(head_dim // 2, dtype=torch.int8, device="cpu")
        if self.mrope_section:
            for dim, offset in ((1, 1), (2, 2)):
                length = self.mrope_section[dim] * 3
                axis[offset:length:3] = dim
        self.axis_of = axis
        self._tables: dict[torch.device, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}

    def tables(self, device: torch.device, max_pos: int = 0):
        """Device tables covering positions [0, max(max_positions, max_pos+1))."""
        cached = self._tables.get(device)
        if cached is None or cached[0].shape[0] <= max_pos:
            n = max(self.max_positions, 1 << int(math.ceil(math.log2(max_pos + 1))))
            p = torch.arange(n, dtype=torch.float32, device="cpu")
            ang = torch.outer(p, self.inv_freq)
            cached = (ang.cos().to(device), ang.sin().to(device), self.axis_of.to(device))
            self._tables[device] = cached
        return cached

    def cos_sin(self, pos: torch.Tensor, dtype: torch.dtype):
        """Eager [T, D] cos/sin for positions ``pos`` of shape [A, T] (HF layout)."""
        inv = self.inv_freq.to(pos.device)
        ang = pos.float().unsqueeze(-1) * inv  # [A, T, D/2]
        axis = self.axis_of.to(pos.device).long()
        if pos.shape[0] > 1:
            ang = ang.gather(0, axis.view(1, 1, -1).expand(1, ang.shape[1], -1)).squeeze(0)
        else:
            ang = ang[0]
        emb = torch.cat([ang, ang], dim=-1)
        return emb.cos().to(dtype), emb.sin().to(dtype)


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, wq, wk, pos, hq, hkv, cache, eps):
        cos_t, sin_t, axis = cache.tables(qkv.device)
        q, k, rstd = _ext.ext().qk_norm_rope_fwd(qkv, hq, hkv, wq, wk, pos, axis, cos_t, sin_t, eps)
        ctx.save_for_backward(qkv, wq, wk, pos, rstd)
        ctx.meta = (hq, hkv, cache)
        ctx.accs = (grad_acc(wq), grad_acc(wk))
        return q, k

    @staticmethod
    def backward(ctx, dq, dk):
        qkv, wq, wk, pos, rstd = ctx.saved_tensors
        hq, hkv, cache = ctx.meta
        cos_t, sin_t, axis = cache.tables(qkv.device, 0)
        dqkv = _QKNormRope.pending_dqkv(qkv)
        dwq, dwk = _ext.ext().qk_norm_rope_bwd(
            dq.contiguous(), dk.contiguous(), qkv, dqkv, hq, hkv, wq, wk, pos, axis, cos_t, sin_t, rstd
        )
        out_w = []
        for w, dw, acc in ((wq, dwq, ctx.accs[0]), (wk, dwk, ctx.accs[1])):
            if acc is not None:
                acc.add_(dw)
                out_w.append(None)
            else:
                out_w.append(dw.to(w.dtype))
        return dqkv, out_w[0], out_w[1], None, None, None, None, None

    @staticmethod
    def pending_dqkv(qkv):
        # The v slice is filled by the attention backward through the same buffer
        # when both run in one fused block; standalone use gets zeros there.
        return torch.zeros_like(qkv)


class _QKNormRopeAttention(torch.autograd.Function):
    """QK-norm + RoPE + varlen flash attention on one ``qkv`` buffer.  The backward writes dV (from the
    attention kernel) and dQ / dK (from the norm/RoPE kernel) straight into one ``dqkv`` buffer, so no
    zero fill, slice copy or gradient sum over ``qkv`` is needed."""

    @staticmethod
    def forward(ctx, qkv, wq, wk, pos, hq, hkv, cache, eps, cu, scale, causal):
        D = cache.head_dim
        cos_t, sin_t, axis = cache.tables(qkv.device)
        ext = _ext.ext()
        q, k, rstd = ext.qk_norm_rope_fwd(qkv, hq, hkv, wq, wk, pos, axis, cos_t, sin_t, eps)
        v = qkv[:, (hq + hkv) * D:].view(qkv.shape[0], hkv, D)
        o, lse = ext.flash_attn_fwd(q, k, v, cu, scale, causal, _ext.status_buffer(q.device).data_ptr())
        # q and k (5/6 of qkv's size) are not kept: the backward recomputes them from qkv in one
        # bandwidth-bound pass, which lets more decoder layers skip activation checkpointing.
        ctx.save_for_backward(qkv, wq, wk, pos, rstd, o, lse, cu)
        ctx.meta = (hq, hkv, cache, scale, causal, float(eps))
        ctx.accs = (grad_acc(wq), grad_acc(wk))
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, wq, wk, pos, rstd, o, lse, cu = ctx.saved_tensors
        hq, hkv, cache, scale, causal, eps = ctx.meta
        D = cache.head_dim
        T = qkv.shape[0]
        ext = _ext.ext()
        cos_f, sin_f, axis_f = cache.tables(qkv.device)
        q, k, _ = ext.qk_norm_rope_fwd(qkv, hq, hkv, wq, wk, pos, axis_f, cos_f, sin_f, eps)
        dqkv = torch.empty_like(qkv)
        v = qkv[:, (hq + hkv) * D:].view(T, hkv, D)
        dk_buf = torch.empty(T, hkv, D, dtype=qkv.dtype, device=qkv.device)
        dq, dk, _ = ext.flash_attn_bwd(do.contiguous(), q, k, v, o, lse, cu, scale, causal,
                                       _ext.status_buffer(q.device).data_ptr(), dk_out=dk_buf,
                                       dv_out=dqkv[:, (hq + hkv) * D:].view(T, hkv, D))
        cos_t, sin_t, axis = cache.tables(qkv.device, 0)
        aq, ak = ctx.accs
        if (aq is not None and ak is not None and aq.is_contiguous() and ak.is_contiguous() and
                aq.dtype == torch.float32 and ak.dtype == torch.float32):
            # norm-weight gradients added into the fp32 accumulators by the kernel itself
            ext.qk_norm_rope_bwd(dq, dk, qkv, dqkv, hq, hkv, wq, wk, pos, axis, cos_t, sin_t, rstd,
                                 dwq_acc=aq, dwk_acc=ak)
            return dqkv, None, None, None, None, None, None, None, None, None, None
        dwq, dwk = ext.qk_norm_rope_bwd(dq, dk, qkv, dqkv, hq, hkv, wq, wk, pos, axis, cos_t, sin_t, rstd)
        out_w = []
        for w, dw, acc in ((wq, dwq, ctx.accs[0]), (wk, dwk, ctx.accs[1])):
            if acc is not None:
                acc.add_(dw)
                out_w.append(None)
            else:
                out_w.append(dw.to(w.dtype))
        return dqkv, out_w[0], out_w[1], None, None, None, None, None, None, None, None


def qk_norm_rope_attention(qkv: torch.Tensor, n_q: int, n_kv: int, wq: torch.Tensor, wk: torch.Tensor,
                           pos: torch.Tensor, cache: "RopeCache", eps: float, cu_seqlens: torch.Tensor,
                           max_seqlen: int, scale: float, causal: bool = True) -> torch.Tensor:
    """``flash_attn_varlen(*qk_norm_rope(qkv), v)`` over packed documents; returns ``o [T, n_q, D]``."""
    D = cache.head_dim
    if not _native(qkv) or D != 128 or qkv.dtype != torch.bfloat16 or qkv.stride(-1) != 1:
        from .attention import flash_attn_varlen

        q, k = qk_norm_rope(qkv, n_q, n_kv, wq, wk, pos, cache, eps)
        v = qkv[:, (n_q + n_kv) * D:].view(-1, n_kv, D)
        return flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen, causal=causal, softmax_scale=scale)
    pos = pos.to(torch.int32).contiguous()
    cu = cu_seqlens.to(device=qkv.device, dtype=torch.int32)
    return _QKNormRopeAttention.apply(qkv, wq, wk, pos, n_q, n_kv, cache, float(eps), cu, float(scale), bool(causal))


def _rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def qk_norm_rope(
    qkv: torch.Tensor,
    n_q: int,
    n_kv: int,
    wq: torch.Tensor,
    wk: torch.Tensor,
    pos: torch.Tensor,
    cache: RopeCache,
    eps: float,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-head RMSNorm of q and k followed by RoPE.

    ``qkv`` is ``[T, (n_q + 2 n_kv) * D]``; ``pos`` is ``[A, T]`` int (A = 1
    for RoPE, 3 for M-RoPE).  Returns ``q [T, n_q, D]`` and ``k [T, n_kv, D]``.
    """
    D = cache.head_dim
    T = qkv.shape[0]
    if not _native(qkv):
        q = qkv[:, : n_q * D].reshape(T, n_q, D)
        k = qkv[:, n_q * D : (n_q + n_kv) * D].reshape(T, n_kv, D)
        q = _rms_norm_eager(q, wq, eps)
        k = _rms_norm_eager(k, wk, eps)
        cos, sin = cache.cos_sin(pos, qkv.dtype)
        cos = cos.unsqueeze(1)
        sin = sin.unsqueeze(1)
        return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin
    if D != 128:
        raise ValueError("qk_norm_rope: the CUDA kernel is specialised for head_dim 128")
    pos = pos.to(torch.int32).contiguous()
    return _QKNormRope.apply(qkv, wq, wk, pos, n_q, n_kv, cache, float(eps))


# ------------------------------------------------------------------- SwiGLU
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        ctx.save_for_backward(gu)
        return _ext.ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dout):
        (gu,) = ctx.saved_tensors
        return _ext.ext().swiglu_bwd(gu, dout.contiguous())


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``gu = [T, 2F]`` (gate columns first)."""
    if not _native(gu):
        g, u = gu.chunk(2, dim=-1)
        return F.silu(g) * u
    return _SwiGLU.apply(gu)


class _SwiGLULinear(torch.autograd.Function):
    """``swiglu(gu) @ w^T`` that keeps only ``gu`` for the backward: the activation (half the size of
    ``gu``) is recomputed there, one bandwidth-bound pass, instead of being held from forward to
    backward.  The memory saved lets more decoder layers skip activation checkpointing."""

    @staticmethod
    def forward(ctx, gu, w):
        gu = gu.contiguous()
        act = _ext.ext().swiglu_fwd(gu)
        y = gemm(act, w)
        ctx.save_for_backward(gu, w)
        ctx.acc = grad_acc(w)
        return y

    @staticmethod
    def backward(ctx, dy):
        gu, w = ctx.saved_tensors
        dy = dy.contiguous()
        act = _ext.ext().swiglu_fwd(gu)
        dw = None
        if ctx.acc is not None or ctx.needs_input_grad[1]:
            dw = _wgrad(dy, act, w, ctx.acc)
        dact = gemm(dy, w, b_mn=True)
        del act
        return _ext.ext().swiglu_bwd(gu, dact), dw


def swiglu_linear(gu: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``linear(swiglu(gu), w)`` (the SwiGLU MLP's down projection) without keeping the activation."""
    if not _native(gu):
        return F.linear(swiglu(gu), w.to(gu.dtype))
    if w.dtype != torch.bfloat16 or gu.dtype != torch.bfloat16:
        return linear(swiglu(gu), w)
    return _SwiGLULinear.apply(gu, w)


# ---------------------------------------------------------------- embedding
class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w, anchor):
        ctx.save_for_backward(ids, w)
        ctx.acc = grad_acc(w)
        return _ext.ext().embedding_fwd(w, ids.reshape(-1).contiguous(),
                                        _ext.status_buffer(w.device).data_ptr()).view(*ids.shape, w.shape[1])

    @staticmethod
    def backward(ctx, dout):
        ids, w = ctx.saved_tensors
        acc = ctx.acc
        dw = None
        if acc is not None:
            _ext.ext().embedding_bwd_(acc, dout.reshape(-1, w.shape[1]).contiguous(), ids.reshape(-1).contiguous())
        elif ctx.needs_input_grad[1]:
            g = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
            _ext.ext().embedding_bwd_(g, dout.reshape(-1, w.shape[1]).contiguous(), ids.reshape(-1).contiguous())
            dw = g.to(w.dtype)
        return None, dw, None


def embedding(ids: torch.Tensor, w: torch.Tensor, anchor: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Row gather ``w[ids]``; ``anchor`` (a tensor requiring grad) forces the backward to run
    when ``w`` itself does not require grad but accumulates through ``_mvp_grad_acc``."""
    if not _native(w):
        return F.embedding(ids, w)
    return _Embedding.apply(ids, w, anchor)


# ------------------------------------------------- fused linear cross-entropy
class _LinearCE(torch.autograd.Function):
    """Chunked LM head + token cross-entropy.

    Without ``grad_hint`` the forward keeps only the row LSEs and the backward recomputes each logits
    chunk.  With ``grad_hint = c`` the caller promises that the loss's gradient will be ``c`` for every
    token (the token-normalised loss with a fixed divisor and no loss guard): the forward then finishes
    each chunk's backward while its logits are still at hand -- softmax minus one-hot in place, the input
    gradient GEMM into a saved ``dh`` and the weight gradient straight into its accumulator -- so the
    logits GEMM runs once instead of twice.  The backward only rescales ``dh`` rows by ``g / c`` (exact
    for any per-token ``g``; the weight gradient needs the promise)."""

    @staticmethod
    def forward(ctx, h, w, labels, chunk, grad_hint):
        T = h.shape[0]
        ext = _ext.ext()
        losses = torch.empty(T, dtype=torch.float32, device=h.device)
        lses = torch.empty(T, dtype=torch.float32, device=h.device)
        ctx.chunk = chunk
        ctx.acc = grad_acc(w)
        ctx.hint = grad_hint
        early = grad_hint is not None
        if early:
            dh = torch.empty_like(h)
            g_hint = torch.full((T,), float(grad_hint), dtype=torch.float32, device=h.device)
            want_dw = ctx.acc is None and ctx.needs_input_grad[1]
            dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device) if want_dw else None
            target = ctx.acc if ctx.acc is not None else dw
            ctx.w_dtype = w.dtype
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            logits = gemm(h[s:e], w)
            loss, lse = ext.ce_fwd(logits, labels[s:e])
            losses[s:e] = loss
            lses[s:e] = lse
            if early:
                ext.ce_bwd_(logits, labels[s:e], lse, g_hint[s:e])
                gemm(logits, w, b_mn=True, out=dh[s:e])
                if target is not None:
                    gemm(logits, h[s:e], a_mn=True, b_mn=True, out=target, accumulate=True)
            del logits
        if early:
            ctx.save_for_backward(dh, dw if dw is not None else torch.empty(0, device=h.device))
        else:
            ctx.save_for_backward(h, w, labels, lses)
        return losses

    @staticmethod
    def backward(ctx, g):
        if ctx.hint is not None:
            dh, dw = ctx.saved_tensors
            ratio = (g.float() / ctx.hint).reshape(-1, 1) if g.numel() > 1 else g.float().reshape(1, 1) / ctx.hint
            dx = (dh.float() * ratio).to(dh.dtype)
            w_grad = dw.to(ctx.w_dtype) if dw.numel() else None
            return dx, w_grad, None, None, None
        h, w, labels, lses = ctx.saved_tensors
        chunk = ctx.chunk
        g = g.float()
        if g.dim() == 0 or g.numel() == 1:
            g = g.reshape(1).expand(h.shape[0])
        g = g.contiguous()
        dh = torch.empty_like(h)
        acc = ctx.acc
        dw = None
        if acc is None and ctx.needs_input_grad[1]:
            dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        target = acc if acc is not None else dw
        for s in range(0, h.shape[0], chunk):
            e = min(h.shape[0], s + chunk)
            logits = gemm(h[s:e], w)
            _ext.ext().ce_bwd_(logits, labels[s:e], lses[s:e], g[s:e])
            gemm(logits, w, b_mn=True, out=dh[s:e])
            if target is not None:
                gemm(logits, h[s:e], a_mn=True, b_mn=True, out=target, accumulate=True)
            del logits
        return dh, (dw.to(w.dtype) if dw is not None else None), None, None, None


def fused_linear_cross_entropy(
    h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, chunk_size: int = 4096,
    grad_hint: Optional[float] = None,
) -> torch.Tensor:
    """Per-token CE of ``h @ w.T`` against ``labels`` (ignore index -100), chunked so the
    full ``[T, V]`` logits never exist; the backward recomputes each logits chunk, unless ``grad_hint``
    (the promised, uniform per-token gradient of the loss) lets the forward finish the backward of each
    chunk right away (see :class:`_LinearCE`)."""
    if not _native(h):
        out = []
        for s in range(0, h.shape[0], chunk_size):
            lg = F.linear(h[s : s + chunk_size], w.to(h.dtype))
            out.append(F.cross_entropy(lg.float(), labels[s : s + chunk_size], ignore_index=-100, reduction="none"))
        return torch.cat(out) if out else h.new_zeros(0, dtype=torch.float32)
    hint = None if grad_hint is None or not torch.is_grad_enabled() else float(grad_hint)
    return _LinearCE.apply(h.contiguous(), w, labels.contiguous(), int(chunk_size), hint)


# ------------------------------------------------------------ optimizer ops
def adamw_step_(
    p: torch.Tensor,
    g: torch.Tensor,
    m: torch.Tensor,
    v: torch.Tensor,
    *,
    lr: float,
    beta1: float,
    beta2: float,
    eps: float,
    weight_decay: float,
    step: int,
    grad_scale: float = 1.0,
    norm_sq: Optional[torch.Tensor] = None,
    max_norm: float = 0.0,
    p_bf16: Optional[torch.Tensor] = None,
) -> None:
    """Decoupled-weight-decay Adam on flat fp32 buffers, mirroring ``torch.optim.AdamW``
    (single-tensor path).  The gradient is multiplied by ``grad_scale`` and, when
    ``norm_sq`` is given, by the clip coefficient ``min(1, max_norm / (sqrt(norm_sq)*grad_scale + 1e-6))``."""
    if not _native(p):
        with torch.no_grad():
            scale = grad_scale
            if norm_sq is not None:
                total = float(norm_sq.sqrt()) * grad_scale
                scale *= min(1.0, max_norm / (total + 1e-6))
            gg = g * scale
            p.mul_(1 - lr * weight_decay)
            m.lerp_(gg, 1 - beta1)
            v.mul_(beta2).addcmul_(gg, gg, value=1 - beta2)
            bc1 = 1 - beta1**step
            bc2 = 1 - beta2**step
            denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
            p.addcdiv_(m, denom, value=-lr / bc1)
            if p_bf16 is not None:
                p_bf16.copy_(p)
        return
    _ext.ext().adamw_step_(
        p, g, m, v, p_bf16, lr, beta1, beta2, eps, weight_decay, int(step), grad_scale, norm_sq, max_norm
    )


# ------------------------------------------------- vision tower (LayerNorm, bias + GELU, RoPE)
def _acc_of(t: torch.Tensor, acc: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """``acc`` if the kernel can add into it directly (contiguous fp32 of ``t``'s size)."""
    if acc is not None and acc.is_contiguous() and acc.dtype == torch.float32 and acc.numel() == t.numel():
        return acc
    return None


def _param_grad(g32: torch.Tensor, p: torch.Tensor, acc: Optional[torch.Tensor], added: bool):
    """Route an fp32 parameter gradient: already added by the kernel, added here, or returned."""
    if added:
        return None
    if acc is not None:
        acc.add_(g32.view_as(acc))
        return None
    return g32.view_as(p).to(p.dtype)


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y, mean, rstd = _ext.ext().layernorm_fwd(x2, w.contiguous(), b.contiguous(), eps)
        ctx.save_for_backward(x2, mean, rstd, w)
        ctx.acc = (grad_acc(w), grad_acc(b))
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, mean, rstd, w = ctx.saved_tensors
        aw, ab = ctx.acc
        kw, kb = _acc_of(w, aw), _acc_of(w, ab)
        dx, dw, db = _ext.ext().layernorm_bwd(dy.reshape(x2.shape).contiguous(), x2, mean, rstd, w.contiguous(),
                                              dw_acc=kw, db_acc=kb)
        return (dx.view(ctx.shape), _param_grad(dw, w, aw, kw is not None), _param_grad(db, w, ab, kb is not None),
                None)


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    """LayerNorm over the last dimension with weight and bias (fp32 statistics, one bf16 rounding).

    On CUDA bf16 input it runs the sm_100a kernel pair; elsewhere ``F.layer_norm``.
    """
    if not _native(x) or x.dtype != torch.bfloat16:
        return F.layer_norm(x, (x.shape[-1],), w.to(x.dtype), b.to(x.dtype), eps)
    return _LayerNorm.apply(x, w.to(x.dtype), b.to(x.dtype), float(eps))


class _BiasGelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, b, tanh_form):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y = _ext.ext().bias_gelu_fwd(x2, b.contiguous(), tanh_form)
        ctx.save_for_backward(x2, b)
        ctx.acc = grad_acc(b)
        ctx.tanh_form = tanh_form
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, b = ctx.saved_tensors
        kb = _acc_of(b, ctx.acc)
        dx, db = _ext.ext().bias_gelu_bwd(dy.reshape(x2.shape).contiguous(), x2, b.contiguous(), ctx.tanh_form,
                                          db_acc=kb)
        return dx.view(ctx.shape), _param_grad(db, b, ctx.acc, kb is not None), None


def bias_gelu(x: torch.Tensor, b: torch.Tensor, approximate: str = "none") -> torch.Tensor:
    """``gelu(x + b)`` with ``approximate`` "tanh" or "none" (erf), the bias add rounded as eager rounds it."""
    if approximate not in ("none", "tanh"):
        raise ValueError(f"bias_gelu: approximate must be 'none' or 'tanh', got {approximate!r}")
    if not _native(x) or x.dtype != torch.bfloat16:
        return F.gelu(x + b.to(x.dtype), approximate=approximate)
    return _BiasGelu.apply(x, b.to(x.dtype), approximate == "tanh")


class _BiasResidual(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, b, x):
        shape = y.shape
        out = _ext.ext().bias_residual_fwd(y.reshape(-1, shape[-1]).contiguous(), b.contiguous(),
                                           x.reshape(-1, shape[-1]).contiguous())
        ctx.save_for_backward(b)
        ctx.acc = grad_acc(b)
        return out.view(shape)

    @staticmethod
    def backward(ctx, dout):
        (b,) = ctx.saved_tensors
        kb = _acc_of(b, ctx.acc)
        db = _ext.ext().bias_grad(dout.reshape(-1, dout.shape[-1]).contiguous(), acc=kb)
        return dout, _param_grad(db, b, ctx.acc, kb is not None), dout


def bias_residual(y: torch.Tensor, b: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """``x + (y + b)``: a bias-free projection's bias add and the residual add in one pass on CUDA bf16.

    Each add rounds to the activation dtype as the two eager adds do; the backward passes the gradient
    through to ``x`` and ``y`` and sums it over rows for ``b`` (into ``b``'s fp32 accumulator when present).
    """
    if not _native(y) or y.dtype != torch.bfloat16:
        return x + (y + b.to(y.dtype))
    return _BiasResidual.apply(y, b.to(y.dtype), x)


class _VisionRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv2, nh, cos, sin, pad_to, bias):
        q, k, v = _ext.ext().vision_rope_fwd(qkv2, nh, cos, sin, pad_to, bias=bias)
        ctx.save_for_backward(cos, sin, bias if bias is not None else torch.empty(0))
        ctx.has_bias = bias is not None
        ctx.acc = grad_acc(bias) if bias is not None else None
        ctx.D = qkv2.shape[1] // (3 * nh)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin, bias = ctx.saved_tensors
        dq, dk, dv = (t.contiguous() if t is not None else None for t in (dq, dk, dv))
        zero = next(t for t in (dq, dk, dv) if t is not None)
        dq, dk, dv = (t if t is not None else torch.zeros_like(zero) for t in (dq, dk, dv))
        dqkv = _ext.ext().vision_rope_bwd(dq, dk, dv, cos, sin, ctx.D)
        db = None
        if ctx.has_bias:  # the bias gradient is the column sum of the pre-rotation gradient
            kb = _acc_of(bias, ctx.acc)
            g32 = _ext.ext().bias_grad(dqkv, acc=kb)
            db = _param_grad(g32, bias, ctx.acc, kb is not None)
        return dqkv, None, None, None, None, db


def vision_rope_pad(qkv: torch.Tensor, nh: int, cos: torch.Tensor, sin: torch.Tensor,
                    pad_to: int = 128, bias: Optional[torch.Tensor] = None
                    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Rotate-half RoPE of the vision tower applied to q and k of a fused ``qkv`` ``[N, 3 * nh * D]``, after
    adding the optional qkv ``bias`` ``[3 * nh * D]`` (rounded to bf16 as a separate add would round it).

    ``cos`` / ``sin`` are ``[N, D / 2]`` fp32 (the rotary angles' cos / sin; each is used for both halves).
    Returns ``q, k, v`` as ``[N, nh, pad_to]`` with columns ``D..pad_to-1`` zero, the layout the
    head_dim-128 attention kernel takes (zero columns leave QK^T and the output's first D columns exact).
    The rotation is computed in fp32 and rounded to the activation dtype once.
    """
    N = qkv.shape[0]
    D = qkv.shape[-1] // (3 * nh)
    if not _native(qkv) or qkv.dtype != torch.bfloat16:
        if bias is not None:
            qkv = qkv + bias.to(qkv.dtype)
        t = qkv.view(N, 3, nh, D)
        c = torch.cat([cos, cos], -1).unsqueeze(1)
        s = torch.cat([sin, sin], -1).unsqueeze(1)
        out = []
        for i in range(2):
            xf = t[:, i].float()
            a, bb = xf.chunk(2, dim=-1)
            out.append((xf * c + torch.cat((-bb, a), -1) * s).to(qkv.dtype))
        out.append(t[:, 2])
        return tuple(F.pad(o, (0, pad_to - D)) for o in out)
    if bias is not None and bias.dtype != torch.bfloat16:
        bias = bias.to(torch.bfloat16)
    return _VisionRope.apply(qkv.reshape(N, -1).contiguous(), int(nh), cos.float().contiguous(),
                             sin.float().contiguous(), int(pad_to), bias.contiguous() if bias is not None else None)


def sumsq(x: torch.Tensor) -> torch.Tensor:
    """Sum of squares of a contiguous fp32/bf16 buffer (fp32 result, deterministic order)."""
    if not _native(x):
        return x.float().pow(2).sum()
    return _ext.ext().sumsq(x.contiguous())


# ------------------------------------------------------------- peer collectives
def peer_reduce_scatter(peer_bufs: list[int], peer_slots: list[int], my_slots: int, rank: int, offset: int,
                        shard: int, seq: int, out: torch.Tensor, scale: float = 1.0,
                        sumsq: Optional[torch.Tensor] = None, timeout_s: float = 10.0) -> None:
    """``out = scale * sum over ranks of buf_r[offset + rank*shard : +shard]`` pulled over NVLink from the
    peers' symmetric buffers, after every rank has published sequence number ``seq`` (bounded wait)."""
    _ext.ext().peer_reduce_scatter(peer_bufs, peer_slots, my_slots, rank, offset, shard, seq, scale, out, sumsq,
                                   _ext.status_buffer(out.device).data_ptr(), int(timeout_s * 1e9))


def peer_gather_shards(peer_bufs: list[int], peer_flags: list[int], rank: int, offset: int, shard: int, epoch: int,
                       out: torch.Tensor, timeout_s: float = 10.0) -> None:
    """``out[r*shard:(r+1)*shard] = bf16 shard r`` read from rank r's symmetric buffer at element ``offset``,
    once every rank has published ``epoch`` (bounded wait): the FSDP parameter gather by pulling."""
    _ext.ext().peer_gather_shards(peer_bufs, peer_flags, offset, shard, epoch, out,
                                  _ext.status_buffer(out.device).data_ptr(), int(timeout_s * 1e9))


def publish_epoch(flag_ptr: int, epoch: int) -> None:
    """Stream-ordered system-scope release of ``epoch`` into this rank's flag (after the kernels before it)."""
    _ext.ext().publish_epoch(int(flag_ptr), int(epoch))


def peer_barrier(peer_slots: list[int], my_slots: int, rank: int, seq: int, timeout_s: float = 10.0) -> None:
    """Stream-ordered device barrier over the peers' signal slots (bounded wait)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    _ext.ext().peer_barrier(peer_slots, my_slots, rank, seq, _ext.status_buffer(dev).data_ptr(), int(timeout_s * 1e9))
