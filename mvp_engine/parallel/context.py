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

Fused ring (``impl: ring`` with ``comm.fused``, the default on CUDA).  No NCCL
call and no ring forwarding: every rank copies its K/V into a symmetric
(peer-mapped) buffer and publishes a sequence number; the attention kernel of
hop s carries extra CTAs that pull rank (r - s - 1)'s K/V block straight from
that rank's memory over NVLink into a local staging buffer while its own CTAs
attend the block of hop s (NVSwitch gives every pair of GPUs full bandwidth,
so the blocks come from their owners, not from the ring neighbour).  In the
backward pass the kernel's epilogue writes each hop's fp32 dK/dV partial
straight into the owner's slot [this rank] of a symmetric accumulator; the
owner then publishes, waits for every rank and sums its slots.  Every wait is
bounded and reports through the status word.

Ulysses (``impl: ulysses``).  An all-to-all turns [2C local tokens, all
heads] into [all T tokens, H/W heads] (chunks put back in sequence order),
the ordinary varlen attention runs over the full sequence for those heads,
and the inverse all-to-all restores the local layout.  Needs H_kv % W == 0.

Fused Ulysses (``impl: ulysses`` with ``comm.fused``).  The all-to-alls
are folded into the kernels that produce the data, so every tile crosses
NVLink once, written straight to where its consumer reads it:

* forward, sequence -> heads: the QKV projection's two-SM GEMM epilogue
  writes each (token, head) element into the symmetric buffer of the rank
  that owns the head, at the token's global row; QK-norm + RoPE then run on
  the full row for this rank's heads;
* forward, heads -> sequence: the attention kernel's epilogue writes each
  output row into the token rank's o_proj input as well as locally;
* backward, sequence -> heads: the o_proj input-gradient GEMM epilogue
  scatters dO to the head ranks;
* backward, heads -> sequence: the attention backward writes dV, and the
  QK-norm/RoPE backward writes dQ / dK, into the token rank's dQKV.

Each scatter is followed by a publish of a sequence number and a bounded
wait for every rank's; the receiving buffers are double-buffered in program
order (the same argument as the fused ring).

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


# ------------------------------------------------------------------ fused ring (NVLink peer pulls)
_WAIT_NS = 10_000_000_000


class _RingPeer:
    """Symmetric buffers and signal slots of one context-parallel group for the fused ring.

    * ``kv[parity]`` [2, L, Hkv, D] bf16 (symmetric): this rank's K/V of one attention call, read by
      every peer.  Uses alternate parity in program order (the same on every rank); a rank starts use
      n only after it pulled every peer's use n-1 block, i.e. after every peer finished use n-2, so
      the buffer it overwrites is no longer read.
    * ``stage[2]`` [2, L, Hkv, D] bf16 (local): the visiting K/V of the current / next hop.
    * ``dkv`` [W, 2, L, Hkv, D] fp32 (symmetric): slot s receives source rank s's dK/dV partial for
      this rank's keys.  Zeroed before this rank publishes its K/V, and peers write into it only
      after they pulled that K/V, so no write of the current use is lost.
    * ``slots`` int64 [8] (symmetric): slot s holds the last sequence number rank s published.
    """

    def __init__(self, cp: "ContextParallel", L: int, Hkv: int, D: int, device) -> None:
        import torch.distributed._symmetric_memory as symm

        self.symm = symm
        group = cp.group if cp.group is not None else dist.group.WORLD
        try:
            symm.enable_symm_mem_for_group(group.group_name)
        except Exception:  # noqa: BLE001 - not needed on newer torch
            pass
        self.group, self.rank, self.world = group, cp.rank, cp.world
        self.shape = (2, L, Hkv, D)
        self.slots = symm.empty(8, dtype=torch.int64, device=device)
        self.slots.zero_()
        n = 2 * L * Hkv * D
        self.kv = [symm.empty(n, dtype=torch.bfloat16, device=device).view(self.shape) for _ in range(2)]
        self.dkv = symm.empty(self.world * n, dtype=torch.float32, device=device).view(self.world, *self.shape)
        torch.cuda.synchronize(device)
        hs = symm.rendezvous(self.slots, group)
        self._handles = [hs] + [symm.rendezvous(t, group) for t in (*self.kv, self.dkv)]
        hs.barrier()
        self.peer_slots = [int(x) for x in hs.buffer_ptrs]
        self.my_slots = int(self.slots.data_ptr())
        self.kv_bases = [[int(x) for x in h.buffer_ptrs] for h in self._handles[1:3]]
        self.dkv_bases = [int(x) for x in self._handles[3].buffer_ptrs]
        self.stage = [torch.empty(self.shape, dtype=torch.bfloat16, device=device) for _ in range(2)]
        self.kv_bytes = n * 2
        self.uses = 0
        self.seq = 0

    def next_seq(self) -> int:
        self.seq += 1
        return self.seq

    def publish_kv(self, k: torch.Tensor, v: torch.Tensor, zero_dkv: bool = False) -> tuple[int, torch.Tensor, list]:
        """Copy (k, v) into this use's symmetric buffer and publish it; returns (seq, buffer, peer bases)."""
        from ..ops import _ext

        parity = self.uses & 1
        self.uses += 1
        buf = self.kv[parity]
        buf[0].copy_(k)
        buf[1].copy_(v)
        if zero_dkv:
            self.dkv.zero_()
        seq = self.next_seq()
        _ext.ext().peer_publish(self.peer_slots, self.my_slots, self.rank, seq, _status(), _WAIT_NS)
        return seq, buf, self.kv_bases[parity]

    def pull_args(self, bases: list, seq: int, hop: int) -> Optional[list]:
        """Copy job of hop ``hop``: rank (r - hop - 1)'s K/V into ``stage[(hop + 1) % 2]``."""
        if hop + 1 >= self.world:
            return None
        src = (self.rank - hop - 1) % self.world
        dst = self.stage[(hop + 1) % 2]
        return [bases[src], dst.data_ptr(), self.kv_bytes, self.my_slots + 8 * src, seq, _WAIT_NS]

    def visiting(self, own: torch.Tensor, hop: int) -> torch.Tensor:
        return own if hop == 0 else self.stage[hop % 2]


def _status() -> int:
    from ..ops import _ext

    return _ext.status_buffer().data_ptr()


def _ring_peer(cp: "ContextParallel", k: torch.Tensor) -> _RingPeer:
    key = (k.shape[0], k.shape[1], k.shape[2])
    pe = cp._peers.get(key)
    if pe is None:
        pe = _RingPeer(cp, k.shape[0], k.shape[1], k.shape[2], k.device)
        cp._peers[key] = pe
    return pe


class _RingAttentionFused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, plan: RingPlan, scale: float, cp: "ContextParallel"):
        from ..ops import _ext

        ext = _ext.ext()
        C = plan.chunk
        q = q.contiguous()
        pe = _ring_peer(cp, k)
        seq, own, bases = pe.publish_kv(k, v)
        o_acc = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        lse_acc = torch.full((q.shape[1], q.shape[0]), float("-inf"), dtype=torch.float32, device=q.device)
        for s, calls in enumerate(plan.hops):
            kv = pe.visiting(own, s)
            pull = pe.pull_args(bases, seq, s)
            for c in calls:
                qs = slice(c.q_half * C, (c.q_half + 1) * C)
                ks = slice(c.k_half * C, (c.k_half + 1) * C)
                o, lse = ext.flash_attn_fwd(q[qs], kv[0, ks], kv[1, ks], c.cu_q, scale, c.causal, _status(),
                                            cu_seqlens_k=c.cu_k, pull=pull)
                pull = None  # the first call of the hop carries the copy
                _merge(o_acc[qs], lse_acc[:, qs], o, lse)
            if pull is not None:  # a hop without calls still moves the next block
                ext.flash_attn_fwd(q[:0], kv[0, :C], kv[1, :C], plan.hops[0][0].cu_q, scale, True, _status(),
                                   cu_seqlens_k=plan.hops[0][0].cu_k, pull=pull)
        out = o_acc.to(q.dtype)
        ctx.save_for_backward(q, k, v, out, lse_acc)
        ctx.plan, ctx.scale, ctx.cp = plan, scale, cp
        return out

    @staticmethod
    def backward(ctx, do):
        from ..ops import _ext

        ext = _ext.ext()
        q, k, v, out, lse = ctx.saved_tensors
        plan, scale, cp = ctx.plan, ctx.scale, ctx.cp
        C = plan.chunk
        do = do.contiguous()
        pe = _ring_peer(cp, k)
        seq, own, bases = pe.publish_kv(k, v, zero_dkv=True)
        L, Hkv, D = k.shape
        row = Hkv * D  # fp32 elements per key row
        slot_bytes = 2 * L * row * 4  # one source's [2, L, Hkv, D] fp32 slot
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        for s, calls in enumerate(plan.hops):
            kv = pe.visiting(own, s)
            pull = pe.pull_args(bases, seq, s)
            owner = (cp.rank - s) % cp.world
            base = pe.dkv_bases[owner] + cp.rank * slot_bytes
            written: set[int] = set()
            for c in calls:
                qs = slice(c.q_half * C, (c.q_half + 1) * C)
                ks = slice(c.k_half * C, (c.k_half + 1) * C)
                off = c.k_half * C * row * 4
                dkv = [base + off, base + L * row * 4 + off, row, int(c.k_half in written)]
                written.add(c.k_half)
                ext.flash_attn_bwd(do[qs], q[qs], kv[0, ks], kv[1, ks], out[qs], lse[:, qs].contiguous(), c.cu_q,
                                   scale, c.causal, _status(), cu_seqlens_k=c.cu_k, pull=pull, dq_accum=dq[qs],
                                   dkv_f32=dkv)
                pull = None
            if pull is not None:
                ext.flash_attn_fwd(q[:0], kv[0, :C], kv[1, :C], plan.hops[0][0].cu_q, scale, True, _status(),
                                   cu_seqlens_k=plan.hops[0][0].cu_k, pull=pull)
        # every rank's partials for this rank's keys are in pe.dkv: publish "written", wait, sum
        dkv = torch.empty(2, L, Hkv, D, dtype=k.dtype, device=k.device)
        ext.peer_slot_sum_f32(pe.dkv, dkv, pe.peer_slots, pe.my_slots, cp.rank, pe.next_seq(), _status(), _WAIT_NS)
        return dq.to(q.dtype), dkv[0], dkv[1], None, None, None


# ------------------------------------------------------------------ fused Ulysses (NVLink scatters)
class _UlyssesPeer:
    """Symmetric receive buffers of the fused Ulysses block, one double-buffered family per scatter."""

    def __init__(self, cp: "ContextParallel", device) -> None:
        import torch.distributed._symmetric_memory as symm

        self.symm = symm
        self.group = cp.group if cp.group is not None else dist.group.WORLD
        try:
            symm.enable_symm_mem_for_group(self.group.group_name)
        except Exception:  # noqa: BLE001 - not needed on newer torch
            pass
        self.rank, self.world, self.device = cp.rank, cp.world, device
        self.slots = symm.empty(8, dtype=torch.int64, device=device)
        self.slots.zero_()
        torch.cuda.synchronize(device)
        h = symm.rendezvous(self.slots, self.group)
        h.barrier()
        self._slot_handle = h
        self.peer_slots = [int(x) for x in h.buffer_ptrs]
        self.my_slots = int(self.slots.data_ptr())
        self.bufs: dict[tuple, list] = {}
        self.uses: dict[str, int] = {}
        self.seq = 0

    def buffer(self, kind: str, shape: tuple[int, ...]) -> tuple[torch.Tensor, list[int]]:
        parity = self.uses.get(kind, 0) & 1
        self.uses[kind] = self.uses.get(kind, 0) + 1
        key = (kind, tuple(shape), parity)
        ent = self.bufs.get(key)
        if ent is None:
            n = 1
            for d in shape:
                n *= int(d)
            t = self.symm.empty(n, dtype=torch.bfloat16, device=self.device)
            torch.cuda.synchronize(self.device)
            h = self.symm.rendezvous(t, self.group)
            ent = [t.view(*shape), [int(x) for x in h.buffer_ptrs], h]
            self.bufs[key] = ent
        return ent[0], ent[1]

    def sync(self) -> None:
        """Publish the next sequence number and wait (bounded, on the device) for every rank's."""
        from ..ops import _ext

        self.seq += 1
        ext = _ext.ext()
        ext.peer_publish(self.peer_slots, self.my_slots, self.rank, self.seq, _status(), _WAIT_NS)
        ext.peer_wait_all(self.peer_slots, self.my_slots, self.rank, self.seq, _status(), _WAIT_NS)


def _grad_into(w: torch.Tensor, dw: torch.Tensor, acc: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if acc is not None:
        acc.add_(dw)
        return None
    return dw.to(w.dtype)


class _UlyssesBlock(torch.autograd.Function):
    """y [L, H] = o_proj(attention(qk_norm_rope(qkv_proj(hn)))) with the four all-to-alls fused.

    ``hn`` [L = 2C, H] are this rank's (zig-zag) tokens.  Saved for backward: ``hn``, the head-layout
    qkv of the full row (local copy), q / k, the attention output and LSE of this rank's heads, and the
    o_proj input (local copy)."""

    @staticmethod
    def forward(ctx, hn, w_qkv, wq, wk, w_o, meta):
        from .. import ops
        from ..ops import _ext

        cp, pctx, Hq, Hkv, D, eps, scale = meta
        ext = _ext.ext()
        W, r = cp.world, cp.rank
        L = hn.shape[0]
        C, T = L // 2, L * W
        hq, hkv = Hq // W, Hkv // W
        pe = cp.ulysses_peer(hn.device)
        # 1. QKV projection; the epilogue scatters every head to its rank at the token's global row
        width = (hq + 2 * hkv) * D
        qh, qh_bases = pe.buffer("qkv_heads", (T, width))
        ext.gemm_ulysses(hn, w_qkv, False, qh_bases, width, r, C, D, [Hq, Hkv, Hkv], _status())
        pe.sync()
        qkv_h = qh.clone()  # the receive buffer is reused two uses later
        # 2. QK-norm + RoPE over the full row for this rank's heads
        pos = cp.full_positions(pctx, T)
        cos_t, sin_t, axis = pctx.rope.tables(hn.device, pctx.max_seqlen)
        q, k, rstd = ext.qk_norm_rope_fwd(qkv_h, hq, hkv, wq, wk, pos, axis, cos_t, sin_t, eps)
        v = qkv_h[:, (hq + hkv) * D:].view(T, hkv, D)
        # 3. attention; the epilogue also writes each output row into the token rank's o_proj input
        oa, oa_bases = pe.buffer("o_tokens", (L, Hq * D))
        route = [W, r, C, Hq * D, r * hq * D, 0, *oa_bases]
        o_h, lse = ext.flash_attn_fwd(q, k, v, pctx.cu_seqlens, scale, True, _status(), route=route)
        pe.sync()
        oa_local = oa.clone()
        # 4. o_proj on this rank's tokens
        y = ops.gemm(oa_local, w_o)
        ctx.save_for_backward(hn, w_qkv, wq, wk, w_o, qkv_h, q, k, o_h, lse, rstd, oa_local, pos)
        ctx.meta = meta
        # gradient accumulators, read here: under activation checkpointing the saved weights are
        # detached aliases without the attribute
        ctx.accs = tuple(ops.grad_acc(t) for t in (w_qkv, wq, wk, w_o))
        return y

    @staticmethod
    def backward(ctx, dy):
        from .. import ops
        from ..ops import _ext

        hn, w_qkv, wq, wk, w_o, qkv_h, q, k, o_h, lse, rstd, oa_local, pos = ctx.saved_tensors
        cp, pctx, Hq, Hkv, D, eps, scale = ctx.meta
        ext = _ext.ext()
        W, r = cp.world, cp.rank
        L = hn.shape[0]
        C, T = L // 2, L * W
        hq, hkv = Hq // W, Hkv // W
        pe = cp.ulysses_peer(hn.device)
        dy = dy.contiguous()
        acc_qkv, acc_q, acc_k, acc_o = ctx.accs
        dwo = ops._wgrad(dy, oa_local, w_o, acc_o)
        # dO to the head ranks: the input-gradient GEMM's epilogue scatters heads
        doh, doh_bases = pe.buffer("do_heads", (T, hq * D))
        ext.gemm_ulysses(dy, w_o, True, doh_bases, hq * D, r, C, D, [Hq, 0, 0], _status())
        pe.sync()
        # attention backward; dV rows go straight to the token ranks' dqkv (v section)
        full = (Hq + 2 * Hkv) * D
        dqkv, dqkv_bases = pe.buffer("dqkv_tokens", (L, full))
        v = qkv_h[:, (hq + hkv) * D:].view(T, hkv, D)
        dq, dk, _ = ext.flash_attn_bwd(doh.view(T, hq, D), q, k, v, o_h, lse, pctx.cu_seqlens, scale, True,
                                       _status(), route=[W, r, C, full, (Hq + Hkv) * D + r * hkv * D, 0,
                                                         *dqkv_bases])
        # QK-norm + RoPE backward; dQ / dK rows go to the token ranks' dqkv (q and k sections)
        cos_t, sin_t, axis = pctx.rope.tables(hn.device, pctx.max_seqlen)
        dwq, dwk = ext.qk_norm_rope_bwd(dq, dk, qkv_h, dqkv, hq, hkv, wq, wk, pos, axis, cos_t, sin_t, rstd,
                                        route=[W, r, C, full, r * hq * D, Hq * D + r * hkv * D, *dqkv_bases])
        pe.sync()
        dhn = ops.gemm(dqkv, w_qkv, b_mn=True)
        dwqkv = ops._wgrad(dqkv, hn, w_qkv, acc_qkv)
        return dhn, dwqkv, _grad_into(wq, dwq, acc_q), _grad_into(wk, dwk, acc_k), dwo, None


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
        self._peers: dict[tuple, Any] = {}

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

    # ---------------------------------------------------------- fused Ulysses block
    def ulysses_fused(self, hn: torch.Tensor, Hq: int, Hkv: int, D: int) -> bool:
        """True when the decoder layer should run its attention block through :class:`_UlyssesBlock`."""
        return (self.impl == "ulysses" and self.world > 1 and D == 128 and Hq % self.world == 0 and
                Hkv % self.world == 0 and hn.shape[0] % 2 == 0 and hn.shape[0] >= 256 and self.use_fused(hn))

    def ulysses_peer(self, device) -> _UlyssesPeer:
        pe = self._peers.get("ulysses")
        if pe is None:
            pe = _UlyssesPeer(self, device)
            self._peers["ulysses"] = pe
        return pe

    def full_positions(self, pctx, total: int) -> torch.Tensor:
        """Per-document positions of the whole row (int32 [1, T]), from the global document boundaries."""
        cached = getattr(pctx, "_cp_full_pos", None)
        if cached is None or cached.shape[-1] != total:
            from ..models.qwen3 import positions_from_cu_seqlens

            cached = positions_from_cu_seqlens(pctx.cu_seqlens, total).to(torch.int32).view(1, total).contiguous()
            pctx._cp_full_pos = cached
        return cached

    def ulysses_block(self, hn, w_qkv, wq, wk, w_o, pctx, Hq: int, Hkv: int, D: int, eps: float,
                      scale: float) -> torch.Tensor:
        meta = (self, pctx, Hq, Hkv, D, float(eps), float(scale))
        return _UlyssesBlock.apply(hn.contiguous(), w_qkv, wq, wk, w_o, meta)

    # ---------------------------------------------------------- attention
    def use_fused(self, q: torch.Tensor) -> bool:
        """Fused NVLink kernels need CUDA bf16 tensors, the native extension and NCCL ranks."""
        if not (self.fused and q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] == 128 and self.world <= 8):
            return False
        from ..ops import _ext

        return _ext.available()

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
            if self.use_fused(q):
                return _RingAttentionFused.apply(q, k, v, self.plan_for(ctx), scale, self)
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
