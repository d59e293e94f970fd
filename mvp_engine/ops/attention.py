"""Varlen (packed-document) attention.

``flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen, causal)`` attends within
each document of a packed stream; grouped-query attention is handled by
mapping query head ``h`` to key/value head ``h // (Hq // Hkv)``.  On CUDA both
passes run the tcgen05 kernels of ``attention_sm100.cu``; on CPU a per-document
loop over ``scaled_dot_product_attention`` gives the same result.

The reference reaches the same computation through HF's
``flash_attention_2`` varlen path with ``cu_seq_lens_q/k`` built in
recipes/qwen3/model/packing/prepare.py:47-91.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import _ext


def _native(t: torch.Tensor) -> bool:
    if not t.is_cuda:
        return False
    return True if _ext.native_required() else _ext.available()


def attention_reference(q, k, v, cu_seqlens, causal=True, softmax_scale=None, return_lse=False):
    """Eager per-document attention in fp32 math (also the test oracle)."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    scale = softmax_scale if softmax_scale is not None else D**-0.5
    out = torch.zeros(T, Hq, D, dtype=q.dtype, device=q.device)
    lse = torch.full((Hq, T), float("-inf"), dtype=torch.float32, device=q.device)
    cu = cu_seqlens.tolist()
    for s, e in zip(cu[:-1], cu[1:]):
        if e <= s:
            continue
        qq = q[s:e].float().transpose(0, 1)  # [H, L, D]
        kk = k[s:e].float().transpose(0, 1).repeat_interleave(rep, 0)
        vv = v[s:e].float().transpose(0, 1).repeat_interleave(rep, 0)
        att = (qq @ kk.transpose(1, 2)) * scale
        if causal:
            L = e - s
            mask = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
            att = att.masked_fill(mask, float("-inf"))
        lse[:, s:e] = torch.logsumexp(att, dim=-1)
        out[s:e] = (att.softmax(-1) @ vv).transpose(0, 1).to(q.dtype)
    return (out, lse) if return_lse else out


class _FlashAttnVarlen(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_seqlen, causal, scale):
        o, lse = _ext.ext().flash_attn_fwd(q, k, v, cu_seqlens, scale, causal, _ext.status_buffer(q.device).data_ptr())
        ctx.save_for_backward(q, k, v, o, lse, cu_seqlens)
        ctx.causal = causal
        ctx.scale = scale
        ctx.max_seqlen = max_seqlen
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, cu = ctx.saved_tensors
        ext = _ext.ext()
        if hasattr(ext, "flash_attn_bwd"):
            dq, dk, dv = ext.flash_attn_bwd(
                do.contiguous(), q, k, v, o, lse, cu, ctx.scale, ctx.causal, _ext.status_buffer(q.device).data_ptr()
            )
            return dq, dk, dv, None, None, None, None
        # Recompute path through autograd on the eager oracle (used only before the
        # native backward kernel is built into the extension).
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_() for t in (q, k, v))
            out = attention_reference(qq, kk, vv, cu, ctx.causal, ctx.scale)
            dq, dk, dv = torch.autograd.grad(out, (qq, kk, vv), do)
        return dq, dk, dv, None, None, None, None


def flash_attn_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    causal: bool = True,
    softmax_scale: Optional[float] = None,
) -> torch.Tensor:
    """Packed-document attention: q [T, Hq, D], k/v [T, Hkv, D] -> [T, Hq, D]."""
    scale = float(softmax_scale) if softmax_scale is not None else q.shape[-1] ** -0.5
    if not _native(q):
        if q.dtype != k.dtype:
            k, v = k.to(q.dtype), v.to(q.dtype)
        return _sdpa_per_doc(q, k, v, cu_seqlens, causal, scale)
    if q.shape[-1] != 128:
        raise ValueError("flash_attn_varlen: the sm_100a kernel is specialised for head_dim 128")
    cu = cu_seqlens.to(device=q.device, dtype=torch.int32)
    return _FlashAttnVarlen.apply(q.contiguous(), k.contiguous() if k.stride(1) != k.shape[2] else k,
                                  v if v.stride(-1) == 1 and v.stride(1) == v.shape[2] else v.contiguous(),
                                  cu, int(max_seqlen), bool(causal), scale)


def _sdpa_per_doc(q, k, v, cu_seqlens, causal, scale):
    T, Hq, D = q.shape
    rep = Hq // k.shape[1]
    outs = []
    for s, e in zip(cu_seqlens[:-1].tolist(), cu_seqlens[1:].tolist()):
        if e <= s:
            continue
        qq = q[s:e].transpose(0, 1).unsqueeze(0)
        kk = k[s:e].transpose(0, 1).repeat_interleave(rep, 0).unsqueeze(0)
        vv = v[s:e].transpose(0, 1).repeat_interleave(rep, 0).unsqueeze(0)
        o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=causal, scale=scale)
        outs.append(o.squeeze(0).transpose(0, 1))
    return torch.cat(outs, 0) if outs else q.new_zeros(q.shape)


# ----------------------------------------------------------------- key-document pairs
def _pair_mask(Lq: int, Lk: int, causal: bool, device) -> Optional[torch.Tensor]:
    """Disallowed (query, key) cells of one document: causal aligned to the document end."""
    if not causal:
        return None
    t = torch.arange(Lq, device=device).view(-1, 1)
    u = torch.arange(Lk, device=device).view(1, -1)
    return u > t + (Lk - Lq)


def attention_pair_reference(q, k, v, cu_q, cu_k, causal, softmax_scale):
    """Oracle for attention of query documents ``cu_q`` against key documents ``cu_k``
    (document d: rows cu_q[d]..cu_q[d+1] see keys cu_k[d]..cu_k[d+1]).  Returns (o, lse [Hq, Tq])."""
    T, Hq, D = q.shape
    rep = Hq // k.shape[1]
    out = torch.zeros(T, Hq, D, dtype=q.dtype, device=q.device)
    lse = torch.full((Hq, T), float("-inf"), dtype=torch.float32, device=q.device)
    for (qs, qe), (ks, ke) in zip(zip(cu_q.tolist()[:-1], cu_q.tolist()[1:]), zip(cu_k.tolist()[:-1], cu_k.tolist()[1:])):
        if qe <= qs or ke <= ks:
            continue
        qq = q[qs:qe].float().transpose(0, 1)
        kk = k[ks:ke].float().transpose(0, 1).repeat_interleave(rep, 0)
        vv = v[ks:ke].float().transpose(0, 1).repeat_interleave(rep, 0)
        att = (qq @ kk.transpose(1, 2)) * softmax_scale
        m = _pair_mask(qe - qs, ke - ks, causal, q.device)
        if m is not None:
            att = att.masked_fill(m, float("-inf"))
        l = torch.logsumexp(att, dim=-1)
        p = torch.exp(att - l.unsqueeze(-1)).nan_to_num(0.0)
        lse[:, qs:qe] = l
        out[qs:qe] = (p @ vv).transpose(0, 1).to(q.dtype)
    return out, lse


def attention_pair_bwd_reference(do, q, k, v, o, lse, cu_q, cu_k, causal, softmax_scale):
    """Gradients of one (query docs, key docs) pair given the softmax normaliser ``lse`` of the
    complete attention (so per-pair results add up to the full gradient)."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    dq = torch.zeros(T, Hq, D, dtype=torch.float32, device=q.device)
    dk = torch.zeros(k.shape[0], Hkv, D, dtype=torch.float32, device=q.device)
    dv = torch.zeros_like(dk)
    delta = (do.float() * o.float()).sum(-1).transpose(0, 1)  # [Hq, T]
    for (qs, qe), (ks, ke) in zip(zip(cu_q.tolist()[:-1], cu_q.tolist()[1:]), zip(cu_k.tolist()[:-1], cu_k.tolist()[1:])):
        if qe <= qs or ke <= ks:
            continue
        qq = q[qs:qe].float().transpose(0, 1)
        kk = k[ks:ke].float().transpose(0, 1).repeat_interleave(rep, 0)
        vv = v[ks:ke].float().transpose(0, 1).repeat_interleave(rep, 0)
        dd = do[qs:qe].float().transpose(0, 1)
        s = (qq @ kk.transpose(1, 2)) * softmax_scale
        m = _pair_mask(qe - qs, ke - ks, causal, q.device)
        p = torch.exp(s - lse[:, qs:qe].unsqueeze(-1))
        if m is not None:
            p = p.masked_fill(m, 0.0)
        dp = dd @ vv.transpose(1, 2)
        ds = p * (dp - delta[:, qs:qe].unsqueeze(-1)) * softmax_scale
        dq[qs:qe] += (ds @ kk).transpose(0, 1)
        gk = (ds.transpose(1, 2) @ qq).view(Hkv, rep, ke - ks, D).sum(1)
        gv = (p.transpose(1, 2) @ dd).view(Hkv, rep, ke - ks, D).sum(1)
        dk[ks:ke] += gk.transpose(0, 1)
        dv[ks:ke] += gv.transpose(0, 1)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def attention_pair_fwd(q, k, v, cu_q, cu_k, causal, softmax_scale):
    """(o, lse) of ``q`` against a separate key stream (tcgen05 kernel on CUDA)."""
    if _native(q):
        return _ext.ext().flash_attn_fwd(q, k, v, cu_q, softmax_scale, causal, _ext.status_buffer(q.device).data_ptr(),
                                         cu_seqlens_k=cu_k)
    return attention_pair_reference(q, k, v, cu_q, cu_k, causal, softmax_scale)


def attention_pair_bwd(do, q, k, v, o, lse, cu_q, cu_k, causal, softmax_scale):
    if _native(q):
        return _ext.ext().flash_attn_bwd(do.contiguous(), q, k, v, o, lse, cu_q, softmax_scale, causal,
                                         _ext.status_buffer(q.device).data_ptr(), cu_seqlens_k=cu_k)
    return attention_pair_bwd_reference(do, q, k, v, o, lse, cu_q, cu_k, causal, softmax_scale)


def attention_any_head_dim(q, k, v, cu_seqlens, max_seqlen, causal, softmax_scale=None):
    """Varlen attention for head_dim <= 128 on CUDA bf16: zero-padding q/k/v to 128 leaves QK^T and the
    softmax unchanged and the padded output columns zero, so the head_dim-128 kernel computes it exactly."""
    D = q.shape[-1]
    scale = softmax_scale if softmax_scale is not None else D**-0.5
    if q.is_cuda and D < 128 and q.dtype == torch.bfloat16:
        pad = 128 - D
        q, k, v = (F.pad(t, (0, pad)) for t in (q, k, v))
        return flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen, causal=causal, softmax_scale=scale)[..., :D]
    return flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen, causal=causal, softmax_scale=scale)
