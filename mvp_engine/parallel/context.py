"""Context parallelism: ring attention and Ulysses over the ``context`` mesh dimension.

The reference has no context parallelism (only a ``cp`` role name,
mvp_engine/distributed/parallel_mesh.py:21); this module adds it.

Sequence layout (both variants).  One packed row of T tokens is cut into
2W chunks of C = T / 2W tokens for W context ranks; rank r keeps chunks
``r`` and ``2W-1-r`` (zig-zag), which gives every rank the same amount of
causal attention work.  Labels are shifted over the whole row before the
cut, per-document positions are computed over the whole row, and the
document boundaries (``cu_seq_lens_q``) stay global; every layer except
attention works on the local 2C tokens unchanged.

Ring (``impl: ring``).  Each rank attends its two query chunks to the key /
value chunks of every rank, passing K/V one step around the ring per hop
(P2P send/recv overlapped with the attention of the current hop).  A
(query chunk a, key chunk b) pair is skipped when b > a, causal when b == a
and full (documents only) when b < a, so with the zig-zag layout every hop
after the first costs exactly two full-chunk attentions.  Partial results
are merged with their log-sum-exp.  The backward pass re-circulates K/V and
sends each hop's dK/dV partial sums along with them, so after W hops every
rank holds the complete dK/dV of its own chunks.

Ulysses (``impl: ulysses``).  An all-to-all turns [2C local tokens, all
heads] into [all T tokens, H/W heads] (chunks put back in sequence order),
the ordinary varlen attention runs over the full sequence for those heads,
and the inverse all-to-all restores the local layout.  Needs H_kv % W == 0.

Gradient reduction and token counting span data x context ranks
(``ParallelMesh.dp_cp``); the context ranks of a group read the same samples.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..ops.attention import attention_pair_bwd, attention_pair_fwd, flash_attn_varlen


# ------------------------------------------------------------------ planning
def zigzag_chunks(rank: int, world: int) -> tuple[int, int]:
    return rank, 2 * world - 1 - rank


def _clip_cu(cu: list[int], lo: int, hi: int) -> list[int]:
    return [min(max(c, lo), hi) - lo for c in cu]


@dataclass
class PairCall:
    q_half: int  # 0 / 1: which local query chunk
    k_half: int  # 0 / 1: which chunk of the visiting K/V block
    causal: bool
    cu_q: torch.Tensor
    cu_k: torch.Tensor


@dataclass
class RingPlan:
    """Per-hop attention calls of one rank for one packed row (hop s holds rank (r - s) mod W's K/V)."""

    chunk: int
    hops: list[list[PairCall]] = field(default_factory=list)


def build_ring_plan(cu_global: list[int], rank: int, world: int, total: int, device) -> RingPlan:
    C = total // (2 * world)
    mine = zigzag_chunks(rank, world)
    plan = RingPlan(chunk=C)
    cache: dict[tuple[int, int], torch.Tensor] = {}

    def cu_of(c: int) -> torch.Tensor:
        key = (c, 0)
        if key not in cache:
            cache[key] = torch.tensor(_clip_cu(cu_global, c * C, (c + 1) * C), dtype=torch.int32, device=device)
        return cache[key]

    for s in range(world):
        src = (rank - s) % world
        theirs = zigzag_chunks(src, world)
        calls = []
        for qh, a in enumerate(mine):
            for kh, b in enumerate(theirs):
                if b > a:
                    continue
                calls.append(PairCall(qh, kh, b == a, cu_of(a), cu_of(b)))
        plan.hops.append(calls)
    return plan


# ------------------------------------------------------------------ ring attention
def _merge(o_acc: torch.Tensor, lse_acc: torch.Tensor, o: torch.Tensor, lse: torch.Tensor) -> None:
    """In place: (o_acc, lse_acc) <- softmax-weighted merge with a partial (o, lse); o_acc fp32 [L,H,D], lse [H,L]."""
    new = torch.logaddexp(lse_acc, lse)
    safe = torch.where(torch.isfinite(new), new, torch.zeros_like(new))
    w_old = torch.where(torch.isfinite(lse_acc), torch.exp(lse_acc - safe), torch.zeros_like(lse_acc))
    w_new = torch.where(torch.isfinite(lse), torch.exp(lse - safe), torch.zeros_like(lse))
    o_acc.mul_(w_old.transpose(0, 1).unsqueeze(-1)).add_(o.float() * w_new.transpose(0, 1).unsqueeze(-1))
    lse_acc.copy_(new)


def _ring_exchange(send: torch.Tensor, recv: torch.Tensor, group, rank: int, world: int):
    nxt = dist.get_global_rank(group, (rank + 1) % world) if group is not None else (rank + 1) % world
    prv = dist.get_global_rank(group, (rank - 1) % world) if group is not None else (rank - 1) % world
    ops = [dist.P2POp(dist.isend, send, nxt, group), dist.P2POp(dist.irecv, recv, prv, group)]
    return dist.batch_isend_irecv(ops)


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, plan: RingPlan, scale: float, cp: "ContextParallel"):
        C = plan.chunk
        q = q.contiguous()
        kv = torch.stack([k, v])  # [2, 2C, Hkv, D]: the block that travels
        o_acc = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        lse_acc = torch.full((q.shape[1], q.shape[0]), float("-inf"), dtype=torch.float32, device=q.device)
        for s, calls in enumerate(plan.hops):
            reqs, nxt = None, None
            if s + 1 < cp.world:
                nxt = torch.empty_like(kv)
                reqs = _ring_exchange(kv, nxt, cp.group, cp.rank, cp.world)
            for c in calls:
                qs = slice(c.q_half * C, (c.q_half + 1) * C)
                ks = slice(c.k_half * C, (c.k_half + 1) * C)
                o, lse = attention_pair_fwd(q[qs], kv[0, ks], kv[1, ks], c.cu_q, c.cu_k, c.causal, scale)
                _merge(o_acc[qs], lse_acc[:, qs], o, lse)
            if reqs is not None:
                for r in reqs:
                    r.wait()
                kv = nxt
        out = o_acc.to(q.dtype)
        ctx.save_for_backward(q, k, v, out, lse_acc)
        ctx.plan, ctx.scale, ctx.cp = plan, scale, cp
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        plan, scale, cp = ctx.plan, ctx.scale, ctx.cp
        C = plan.chunk
        do = do.contiguous()
        kv = torch.stack([k, v])
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        dkv = torch.zeros(kv.shape, dtype=torch.float32, device=q.device)  # accumulator of the visiting block
        for s, calls in enumerate(plan.hops):
            reqs, nxt = None, None
            if s + 1 < cp.world:
                nxt = torch.empty_like(kv)
                reqs = _ring_exchange(kv, nxt, cp.group, cp.rank, cp.world)
            for c in calls:
                qs = slice(c.q_half * C, (c.q_half + 1) * C)
                ks = slice(c.k_half * C, (c.k_half + 1) * C)
                gq, gk, gv = attention_pair_bwd(do[qs], q[qs], kv[0, ks], kv[1, ks], out[qs], lse[:, qs].contiguous(),
                                                c.cu_q, c.cu_k, c.causal, scale)
                dq[qs] += gq.float()
                dkv[0, ks] += gk.float()
                dkv[1, ks] += gv.float()
            # The accumulator follows its K/V block one step around the ring (the last step
            # brings every block's sums home).
            home = torch.empty_like(dkv)
            for r in _ring_exchange(dkv, home, cp.group, cp.rank, cp.world):
                r.wait()
            dkv = home
            if reqs is not None:
                for r in reqs:
                    r.wait()
                kv = nxt
        return dq.to(q.dtype), dkv[0].to(k.dtype), dkv[1].to(v.dtype), None, None, None


# ------------------------------------------------------------------ Ulysses
def _seq_order(recv: torch.Tensor, world: int) -> torch.Tensor:
    """[W, 2, C, h, D] (per source rank, its two zig-zag chunks) -> [T, h, D] in sequence order."""
    first = recv[:, 0]  # chunks 0..W-1
    second = recv[:, 1].flip(0)  # chunks W..2W-1
    full = torch.cat([first, second], dim=0)
    return full.reshape(-1, *recv.shape[-2:])


def _zigzag_order(full: torch.Tensor, world: int) -> torch.Tensor:
    """Inverse of ``_seq_order``: [T, h, D] -> [W, 2, C, h, D]."""
    g = full.reshape(2 * world, -1, *full.shape[-2:])
    return torch.stack([g[:world], g[world:].flip(0)], dim=1)


class _SeqToHeads(torch.autograd.Function):
    """[2C, H, D] local tokens, all heads -> [T, H/W, D] all tokens, this rank's heads."""

    @staticmethod
    def forward(ctx, x, cp: "ContextParallel"):
        ctx.cp = cp
        return _seq_to_heads(x, cp)

    @staticmethod
    def backward(ctx, g):
        return _heads_to_seq(g.contiguous(), ctx.cp), None


class _HeadsToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cp: "ContextParallel"):
        ctx.cp = cp
        return _heads_to_seq(x, cp)

    @staticmethod
    def backward(ctx, g):
        return _seq_to_heads(g.contiguous(), ctx.cp), None


def _seq_to_heads(x: torch.Tensor, cp: "ContextParallel") -> torch.Tensor:
    W = cp.world
    L, H, D = x.shape
    send = x.reshape(2, L // 2, W, H // W, D).permute(2, 0, 1, 3, 4).contiguous()  # [W(dest), 2, C, h, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=cp.group)
    return _seq_order(recv, W)


def _heads_to_seq(y: torch.Tensor, cp: "ContextParallel") -> torch.Tensor:
    W = cp.world
    send = _zigzag_order(y, W).contiguous()  # [W(dest), 2, C, h, D]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=cp.group)
    _, two, C, h, D = recv.shape
    return recv.permute(1, 2, 0, 3, 4).reshape(two * C, W * h, D)  # heads of source rank j are group j


# ------------------------------------------------------------------ runtime
class ContextParallel:
    """Context-parallel runtime attached to a model (``model._mvp_cp``)."""

    def __init__(self, group: Optional[dist.ProcessGroup], impl: str = "ring", fused: bool = False) -> None:
        if impl not in ("ring", "ulysses"):
            raise ValueError(f"context_parallel.impl must be 'ring' or 'ulysses', got {impl!r}")
        self.group = group
        self.impl = impl
        self.fused = fused
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0

    # ---------------------------------------------------------- batch sharding
    def local_indices(self, total: int) -> torch.Tensor:
        if total % (2 * self.world):
            raise ValueError(f"context parallel needs the packed length ({total}) divisible by 2 x {self.world}")
        C = total // (2 * self.world)
        a, b = zigzag_chunks(self.rank, self.world)
        return torch.cat([torch.arange(a * C, (a + 1) * C), torch.arange(b * C, (b + 1) * C)])

    def shard_batch(self, batch: dict[str, Any], *, ignore_index: int = -100) -> dict[str, Any]:
        """Cut one collated packed row to this rank's zig-zag chunks (host tensors).

        ``labels`` are replaced by ``shift_labels`` (already shifted over the whole row),
        per-document ``position_ids`` are taken from the whole row, ``cu_seq_lens_q`` stays
        global, and ``total_tokens`` / ``effective_tokens`` become this rank's counts.
        """
        from ..kit.llm.data.collator import varlen_metadata

        ids = batch["input_ids"]
        if ids.dim() != 2 or ids.shape[0] != 1:
            raise ValueError("context parallel expects one packed row per micro-batch (batch_size 1)")
        T = ids.shape[1]
        idx = self.local_indices(T)
        out = dict(batch)
        seg = batch.get("pack_segment_ids")
        if seg is None:
            seg = torch.ones_like(ids)
        if "cu_seq_lens_q" not in batch or "position_ids" not in batch:
            cu, mx, pos = varlen_metadata(seg.cpu())
            out.setdefault("cu_seq_lens_q", cu)
            out.setdefault("max_length_q", mx)
            out.setdefault("position_ids", pos)
        pos = out["position_ids"]
        out["position_ids"] = pos[..., idx]
        labels = batch["labels"]
        shifted = F.pad(labels, (0, 1), value=ignore_index)[..., 1:]
        out["shift_labels"] = shifted[:, idx]
        out.pop("labels", None)
        out["input_ids"] = ids[:, idx]
        out["pack_segment_ids"] = seg[:, idx]
        if "attention_mask" in out:
            out["attention_mask"] = out["attention_mask"][:, idx]
        out["total_tokens"] = int((seg[:, idx] > 0).sum()) if batch.get("pack_segment_ids") is not None else len(idx)
        out["effective_tokens"] = int(out["shift_labels"].ne(ignore_index).sum())
        out["cp_total_tokens"] = T
        return out

    # ---------------------------------------------------------- attention
    def plan_for(self, ctx) -> RingPlan:
        cached = getattr(ctx, "_cp_plan", None)
        if cached is None:
            cu = ctx.cu_seqlens.tolist()
            cached = build_ring_plan(cu, self.rank, self.world, int(cu[-1]), ctx.cu_seqlens.device)
            ctx._cp_plan = cached
        return cached

    def attention(self, q, k, v, ctx, scale: float) -> torch.Tensor:
        if self.world == 1:
            return flash_attn_varlen(q, k, v, ctx.cu_seqlens, ctx.max_seqlen, causal=ctx.causal, softmax_scale=scale)
        if self.impl == "ring":
            return _RingAttention.apply(q, k, v, self.plan_for(ctx), scale, self)
        Hq, Hkv = q.shape[1], k.shape[1]
        if Hq % self.world or Hkv % self.world:
            raise ValueError(f"Ulysses needs query ({Hq}) and key/value ({Hkv}) heads divisible by {self.world}")
        qh = _SeqToHeads.apply(q, self)
        kh = _SeqToHeads.apply(k, self)
        vh = _SeqToHeads.apply(v, self)
        o = flash_attn_varlen(qh.contiguous(), kh.contiguous(), vh.contiguous(), ctx.cu_seqlens, ctx.max_seqlen,
                              causal=ctx.causal, softmax_scale=scale)
        return _HeadsToSeq.apply(o, self)


def attach_context_parallel(model: torch.nn.Module, parallel_mesh, impl: str = "ring", fused: bool = False):
    """Attach a :class:`ContextParallel` runtime over the mesh's ``cp`` group to ``model``."""
    cp = ContextParallel(parallel_mesh.cp.group, impl=impl, fused=fused)
    model._mvp_cp = cp
    return cp


def context_parallel_of(model: torch.nn.Module) -> Optional[ContextParallel]:
    m = getattr(model, "module", model)
    return getattr(m, "_mvp_cp", None) or getattr(model, "_mvp_cp", None)


def maybe_shard_batch(model: torch.nn.Module, batch: dict[str, Any]) -> dict[str, Any]:
    """Recipe hook: cut the batch for context parallelism when the model has a CP runtime."""
    cp = context_parallel_of(model)
    if cp is None or cp.world == 1:
        return batch
    return cp.shard_batch(batch)
