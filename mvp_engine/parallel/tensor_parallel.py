"""Native tensor parallelism (Megatron layout) for the engine's Qwen3 decoder.

Reference counterpart: DTensor ``parallelize_module`` plans with
``ColwiseParallel`` / ``RowwiseParallel`` / ``SequenceParallel``
(mvp_engine/distributed/tp.py:41-107).  Here the decoder layer itself calls two
collectives per sub-block and the weights are plain local shards:

* column-parallel: fused q/k/v rows (heads ``r*Hq/tp ..``, kv heads
  ``r*Hkv/tp ..``) and fused gate/up rows (``r*F/tp ..`` of each);
* row-parallel: o_proj and down_proj columns;
* replicated: norms, embedding, LM head (sharded only by the data-parallel
  runtime).

With ``sequence_parallel`` the residual stream, the norms, the embedding and
the loss work on a contiguous 1/tp slice of the tokens; entering a
column-parallel GEMM all-gathers the sequence and leaving a row-parallel GEMM
reduce-scatters it (backward: the reverse).  Without it, activations are
replicated; entering is the identity (backward: all-reduce) and leaving is an
all-reduce.  Replicated weights whose gradient each rank only sees part of
(all of them under sequence parallelism; the per-head QK-norm weights always)
are tagged ``_mvp_tp_partial`` and summed over the tensor group before the
data-parallel reduction.
"""

from __future__ import annotations

from typing import Any, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


def _ag_seq(x: torch.Tensor, group, world: int) -> torch.Tensor:
    out = torch.empty((x.shape[0] * world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _rs_seq(x: torch.Tensor, group, world: int) -> torch.Tensor:
    out = torch.empty((x.shape[0] // world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


def _ar(x: torch.Tensor, group) -> torch.Tensor:
    x = x.contiguous().clone()
    dist.all_reduce(x, group=group)
    return x


class _Enter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp: "TensorParallel"):
        ctx.tp = tp
        return _ag_seq(x, tp.group, tp.world) if tp.sequence_parallel else x

    @staticmethod
    def backward(ctx, g):
        tp = ctx.tp
        return (_rs_seq(g, tp.group, tp.world) if tp.sequence_parallel else _ar(g, tp.group)), None


class _Exit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp: "TensorParallel"):
        ctx.tp = tp
        return _rs_seq(x, tp.group, tp.world) if tp.sequence_parallel else _ar(x, tp.group)

    @staticmethod
    def backward(ctx, g):
        tp = ctx.tp
        return (_ag_seq(g, tp.group, tp.world) if tp.sequence_parallel else g), None


class TensorParallel:
    def __init__(self, group: Optional[dist.ProcessGroup], sequence_parallel: bool = True, fused: bool = False):
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.sequence_parallel = bool(sequence_parallel)
        self.fused = fused

    @property
    def peer(self) -> "_PeerTP":
        p = getattr(self, "_peer", None)
        if p is None:
            p = self._peer = _PeerTP(self)
        return p

    def column_linear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """Column-parallel GEMM of the (sequence-sharded) input: the all-gather is fused with the GEMM
        over NVLink when possible (``fused``, sequence parallel, token count a multiple of 256 x tp)."""
        from .. import ops

        if _fused_ok(self, x, w, x.shape[0] * self.world):
            return _AGLinear.apply(x, w, self)
        return ops.linear(self.enter(x), w)

    def row_linear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """Row-parallel GEMM whose partial sums are reduce-scattered along the sequence.

        The routed-epilogue version (GEMM writes each row block into its owner's slots, owners sum)
        measured slower than GEMM + NCCL reduce-scatter on 2 GPUs (0.29 vs 0.24 ms for a
        4096 x 5120 x 5120 o_proj), so it is used only with MVP_TP_FUSED_ROW=1."""
        from .. import ops

        if _FUSED_ROW and _fused_ok(self, x, w, x.shape[0]):
            return _RSLinear.apply(x, w, self)
        return self.exit(ops.linear(x, w))

    def enter(self, x: torch.Tensor) -> torch.Tensor:
        """Input of a column-parallel GEMM."""
        return _Enter.apply(x, self)

    def exit(self, x: torch.Tensor) -> torch.Tensor:
        """Output (partial sums) of a row-parallel GEMM."""
        return _Exit.apply(x, self)

    def seq_slice(self, T: int) -> slice:
        if not self.sequence_parallel:
            return slice(0, T)
        if T % self.world:
            raise ValueError(f"sequence parallel needs the token count ({T}) divisible by tp={self.world}")
        n = T // self.world
        return slice(self.rank * n, (self.rank + 1) * n)


def _shard_rows(t: torch.Tensor, parts: list[tuple[int, int]]) -> torch.Tensor:
    return torch.cat([t[a:b] for a, b in parts], dim=0)


def _replace(mod: nn.Module, name: str, dim: int, start: int, stop: int) -> None:
    """Replace ``mod.<name>`` by its ``[start, stop)`` slice along ``dim`` and record the slice
    (``_mvp_tp_slice`` = full shape, dim, start, stop).  The data-parallel runtime uses it twice: a
    parameter still on the meta device is initialised as the full tensor and then cut, so a tensor-parallel
    model starts from exactly the weights of the unsharded one (initialising the slice by itself would give
    every rank the same values); and checkpoints store the full logical tensor, assembled from the tensor
    ranks' slices, under the parameter's name."""
    p = getattr(mod, name)
    if getattr(p, "_mvp_tp_slice", None) is not None:  # one slice per parameter is all that is recorded
        raise RuntimeError(f"{name} is already tensor-parallel sharded")
    value = p.narrow(dim, start, stop - start)
    meta = value.device.type == "meta"
    new = nn.Parameter(value if meta else value.detach().clone(), requires_grad=p.requires_grad)
    new._mvp_tp_sharded = True
    new._mvp_tp_slice = (tuple(p.shape), dim, start, stop)
    setattr(mod, name, new)


def apply_native_tensor_parallel(model: nn.Module, parallel_mesh: Any = None, *, group=None,
                                 sequence_parallel: bool = True, fused: bool = False) -> TensorParallel:
    """Shard the Qwen3 decoder layers of ``model`` in place over the tensor group and attach the
    runtime as ``model._mvp_tp``; returns it."""
    from ..models.qwen3 import Qwen3DecoderLayer

    if sequence_parallel and not getattr(model, "supports_sequence_parallel", False):
        raise ValueError(f"{type(model).__name__} does not implement sequence parallelism (the token slicing around "
                         "its embedding and loss); use tensor parallelism without it")
    grp = group if group is not None else parallel_mesh.tp.group
    tp = TensorParallel(grp, sequence_parallel=sequence_parallel, fused=fused)
    W, r = tp.world, tp.rank
    layers = [m for m in model.modules() if isinstance(m, Qwen3DecoderLayer)]
    if not layers:
        raise ValueError(f"native tensor parallelism shards Qwen3 decoder layers; {type(model).__name__} has none")
    for layer in layers:
        a, m = layer.self_attn, layer.mlp
        Hq, Hkv, D = a.num_heads, a.num_kv_heads, a.head_dim
        if Hq % W or Hkv % W:
            raise ValueError(f"tensor parallel {W} needs query ({Hq}) and key/value ({Hkv}) heads divisible by it")
        hq, hkv = Hq // W, Hkv // W
        _replace(a.q_proj, "weight", 0, r * hq * D, (r + 1) * hq * D)
        _replace(a.k_proj, "weight", 0, r * hkv * D, (r + 1) * hkv * D)
        _replace(a.v_proj, "weight", 0, r * hkv * D, (r + 1) * hkv * D)
        _replace(a.o_proj, "weight", 1, r * hq * D, (r + 1) * hq * D)
        F = m.gate_proj.weight.shape[0]
        if F % W:
            raise ValueError(f"tensor parallel {W} needs the FFN width ({F}) divisible by it")
        f = F // W
        _replace(m.gate_proj, "weight", 0, r * f, (r + 1) * f)
        _replace(m.up_proj, "weight", 0, r * f, (r + 1) * f)
        _replace(m.down_proj, "weight", 1, r * f, (r + 1) * f)
        a.num_heads, a.num_kv_heads = hq, hkv
        a.q_norm.weight._mvp_tp_partial = True  # per-head norms see only this rank's heads
        a.k_norm.weight._mvp_tp_partial = True
        layer._tp = tp
    if sequence_parallel:
        for p in model.parameters():
            if not getattr(p, "_mvp_tp_sharded", False):
                p._mvp_tp_partial = True
    model._mvp_tp = tp
    return tp


def tensor_parallel_of(model: nn.Module) -> Optional[TensorParallel]:
    m = getattr(model, "module", model)
    return getattr(m, "_mvp_tp", None) or getattr(model, "_mvp_tp", None)


# ------------------------------------------------------------------ fused NVLink path
class _PeerTP:
    """Symmetric (peer-mapped) buffers and signal slots of one tensor-parallel group.

    Two buffer kinds, each double-buffered and used alternately in program order (the same on every
    rank): ``gather`` [T, H] receives every rank's row slice (pushed by the owners), ``slots``
    [W, T/W, H] receives every source rank's routed partial rows.  A use of a buffer is fully consumed
    before the op returns, and a rank only writes a peer's buffer after seeing that peer publish a
    later sequence number, so a buffer is never overwritten while its owner still reads it.
    """

    def __init__(self, tp: "TensorParallel") -> None:
        import torch.distributed._symmetric_memory as symm

        self.tp = tp
        self.symm = symm
        self.group = tp.group
        try:
            symm.enable_symm_mem_for_group(self.group.group_name)
        except Exception:  # noqa: BLE001 - not needed on newer torch
            pass
        dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.slots = symm.empty(8, dtype=torch.int64, device=dev)
        self.slots.zero_()
        torch.cuda.synchronize(dev)
        h = symm.rendezvous(self.slots, self.group)
        h.barrier()
        self.slot_handle = h
        self.peer_slots = [int(x) for x in h.buffer_ptrs]
        self.my_slots = int(self.slots.data_ptr())
        self.bufs: dict[tuple, list] = {}
        self.uses: dict[str, int] = {}
        self.seq = 0

    def next_seq(self) -> int:
        self.seq += 1
        return self.seq

    def buffer(self, kind: str, shape: tuple[int, ...]) -> tuple[torch.Tensor, list[int]]:
        """(local buffer, every rank's base address) of the next use of ``kind``."""
        parity = self.uses.get(kind, 0) & 1
        self.uses[kind] = self.uses.get(kind, 0) + 1
        key = (kind, tuple(shape), parity)
        ent = self.bufs.get(key)
        if ent is None:
            t = self.symm.empty(int(torch.tensor(shape).prod()), dtype=torch.bfloat16, device=self.device)
            torch.cuda.synchronize(self.device)
            h = self.symm.rendezvous(t, self.group)
            ent = [t.view(*shape), [int(x) for x in h.buffer_ptrs], h]
            self.bufs[key] = ent
        return ent[0], ent[1]


_WAIT_NS = 10_000_000_000
_FUSED_ROW = __import__("os").environ.get("MVP_TP_FUSED_ROW", "0") == "1"


def _status():
    from ..ops import _ext

    return _ext.status_buffer().data_ptr()


def _wgrad(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, acc: Optional[torch.Tensor] = None):
    """dW = dY^T X accumulated into the runtime's fp32 gradient buffer when the weight has one
    (``acc``, captured in the forward: under activation checkpointing the saved weight is a
    detached alias without the attribute)."""
    from .. import ops

    acc = acc if acc is not None else getattr(w, "_mvp_grad_acc", None)
    if acc is not None:
        ops.gemm(dy, x, a_mn=True, b_mn=True, out=acc, accumulate=True)
        return None
    return ops.gemm(dy, x, a_mn=True, b_mn=True, out_dtype=torch.float32).to(w.dtype)


class _AGLinear(torch.autograd.Function):
    """y [T, N] = all_gather_seq(x_sp) @ w^T with the gather pushed over NVLink and consumed slice by slice."""

    @staticmethod
    def forward(ctx, x_sp, w, tp):
        from ..ops import _ext

        pe, W, r = tp.peer, tp.world, tp.rank
        rows, K = x_sp.shape
        T = rows * W
        g, g_bases = pe.buffer("gather", (T, K))
        seq = pe.next_seq()
        ext = _ext.ext()
        ext.peer_push_rows(x_sp.contiguous(), g_bases, r * rows, pe.peer_slots, pe.my_slots, r, seq, _status(),
                           _WAIT_NS)
        y = torch.empty(T, w.shape[0], dtype=torch.bfloat16, device=x_sp.device)
        ext.gemm_pair_tp(g, w, False, y, w.shape[0], pe.my_slots, seq, rows, r * rows, [], 0, 0, _status(), _WAIT_NS)
        ctx.save_for_backward(x_sp, w)
        ctx.tp = tp
        ctx.acc = getattr(w, "_mvp_grad_acc", None)
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops import _ext

        x_sp, w = ctx.saved_tensors
        tp = ctx.tp
        pe, W, r = tp.peer, tp.world, tp.rank
        rows, K = x_sp.shape
        dy = dy.contiguous()
        ext = _ext.ext()
        # dX_sp = reduce_scatter_seq(dY @ W): rows routed to their owners' slots, then summed there
        s, s_bases = pe.buffer("slots", (W, rows, K))
        seq = pe.next_seq()
        ext.gemm_pair_tp(dy, w, True, None, K, 0, 0, 0, 0, [b + r * rows * K * 2 for b in s_bases], rows, 0,
                         _status(), _WAIT_NS)
        dx = torch.empty(rows, K, dtype=torch.bfloat16, device=dy.device)
        ext.peer_slot_reduce(s, dx, pe.peer_slots, pe.my_slots, r, seq, _status(), _WAIT_NS)
        # dW = dY^T X_full: gather X again (not kept from the forward)
        g, g_bases = pe.buffer("gather", (rows * W, K))
        seq2 = pe.next_seq()
        ext.peer_push_rows(x_sp.contiguous(), g_bases, r * rows, pe.peer_slots, pe.my_slots, r, seq2, _status(),
                           _WAIT_NS)
        ext.peer_wait_all(pe.peer_slots, pe.my_slots, r, seq2, _status(), _WAIT_NS)
        dw = _wgrad(dy, g, w, ctx.acc)
        return dx, dw, None


class _RSLinear(torch.autograd.Function):
    """y_sp [T/W, N] = reduce_scatter_seq(x @ w^T) with output rows routed to their owners in the GEMM epilogue."""

    @staticmethod
    def forward(ctx, x, w, tp):
        from ..ops import _ext

        pe, W, r = tp.peer, tp.world, tp.rank
        T = x.shape[0]
        rows, N = T // W, w.shape[0]
        ext = _ext.ext()
        s, s_bases = pe.buffer("slots", (W, rows, N))
        seq = pe.next_seq()
        x = x.contiguous()
        ext.gemm_pair_tp(x, w, False, None, N, 0, 0, 0, 0, [b + r * rows * N * 2 for b in s_bases], rows, 0,
                         _status(), _WAIT_NS)
        y = torch.empty(rows, N, dtype=torch.bfloat16, device=x.device)
        ext.peer_slot_reduce(s, y, pe.peer_slots, pe.my_slots, r, seq, _status(), _WAIT_NS)
        ctx.save_for_backward(x, w)
        ctx.tp = tp
        ctx.acc = getattr(w, "_mvp_grad_acc", None)
        return y

    @staticmethod
    def backward(ctx, dy_sp):
        from ..ops import _ext

        x, w = ctx.saved_tensors
        tp = ctx.tp
        pe, W, r = tp.peer, tp.world, tp.rank
        rows, N = dy_sp.shape
        ext = _ext.ext()
        g, g_bases = pe.buffer("gather", (rows * W, N))
        seq = pe.next_seq()
        ext.peer_push_rows(dy_sp.contiguous(), g_bases, r * rows, pe.peer_slots, pe.my_slots, r, seq, _status(),
                           _WAIT_NS)
        K = w.shape[1]
        dx = torch.empty(rows * W, K, dtype=torch.bfloat16, device=dy_sp.device)
        ext.gemm_pair_tp(g, w, True, dx, K, pe.my_slots, seq, rows, r * rows, [], 0, 0, _status(), _WAIT_NS)
        dw = _wgrad(g, x, w, ctx.acc)  # the input-grad GEMM above has waited for every slice
        return dx, dw, None


def _fused_ok(tp: "TensorParallel", x: torch.Tensor, w: torch.Tensor, tokens: int) -> bool:
    return (tp.fused and tp.sequence_parallel and x.is_cuda and x.dtype == torch.bfloat16 and
            w.dtype == torch.bfloat16 and tp.world <= 8 and tokens % (tp.world * 256) == 0 and
            w.shape[0] >= 256 and w.shape[1] >= 256 and w.shape[1] % 8 == 0 and tokens >= 256)
