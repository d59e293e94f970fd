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


def _replace(mod: nn.Module, name: str, value: torch.Tensor) -> None:
    p = getattr(mod, name)
    new = nn.Parameter(value.detach().clone() if value.device.type != "meta" else value, requires_grad=p.requires_grad)
    new._mvp_tp_sharded = True
    setattr(mod, name, new)


def apply_native_tensor_parallel(model: nn.Module, parallel_mesh: Any = None, *, group=None,
                                 sequence_parallel: bool = True, fused: bool = False) -> TensorParallel:
    """Shard the Qwen3 decoder layers of ``model`` in place over the tensor group and attach the
    runtime as ``model._mvp_tp``; returns it."""
    from ..models.qwen3 import Qwen3DecoderLayer

    grp = group if group is not None else parallel_mesh.tp.group
    tp = TensorParallel(grp, sequence_parallel=sequence_parallel, fused=fused)
    W, r = tp.world, tp.rank
    for layer in model.modules():
        if not isinstance(layer, Qwen3DecoderLayer):
            continue
        a, m = layer.self_attn, layer.mlp
        Hq, Hkv, D = a.num_heads, a.num_kv_heads, a.head_dim
        if Hq % W or Hkv % W:
            raise ValueError(f"tensor parallel {W} needs query ({Hq}) and key/value ({Hkv}) heads divisible by it")
        hq, hkv = Hq // W, Hkv // W
        _replace(a.q_proj, "weight", a.q_proj.weight[r * hq * D:(r + 1) * hq * D])
        _replace(a.k_proj, "weight", a.k_proj.weight[r * hkv * D:(r + 1) * hkv * D])
        _replace(a.v_proj, "weight", a.v_proj.weight[r * hkv * D:(r + 1) * hkv * D])
        _replace(a.o_proj, "weight", a.o_proj.weight[:, r * hq * D:(r + 1) * hq * D])
        F = m.gate_proj.weight.shape[0]
        if F % W:
            raise ValueError(f"tensor parallel {W} needs the FFN width ({F}) divisible by it")
        f = F // W
        _replace(m.gate_proj, "weight", m.gate_proj.weight[r * f:(r + 1) * f])
        _replace(m.up_proj, "weight", m.up_proj.weight[r * f:(r + 1) * f])
        _replace(m.down_proj, "weight", m.down_proj.weight[:, r * f:(r + 1) * f])
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
