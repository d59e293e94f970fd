"""Native flat-buffer fully-sharded data parallelism.

This is the engine's B200 data-parallel runtime; torch FSDP2 stays available
as the reference-equivalent backend (``parallel.backend_kwargs.impl=torch``,
reference: mvp_engine/distributed/fsdp2.py:50-176).

Layout.  Parameters are grouped into *units*: one per ``_no_split_modules``
block (a decoder layer) plus a root unit with everything else.  A unit owns

* ``full``   the unsharded compute weights, one contiguous buffer in
             ``param_dtype`` (bf16); every parameter becomes a view into it,
             so q/k/v (and gate/up) are adjacent and usable as one fused GEMM
             operand;
* ``grad``   an fp32 buffer of the same layout where weight gradients
             accumulate across micro-batches (the GEMM epilogue adds into it
             directly, see ``mvp_engine.ops``);
* ``master``, ``exp_avg``, ``exp_avg_sq``, ``grad_shard``: this rank's
             contiguous 1/W slice, fp32.

Because shards are contiguous slices of the full layout, the parameter
all-gather is an in-place ``all_gather_into_tensor`` into ``full`` and the
gradient reduce-scatter reads ``grad`` as is: no copy-in / copy-out kernels.
The optimizer writes its bf16 output straight into this rank's slice of
``full``.  By default full weights stay resident between steps, so each
parameter crosses NVLink once per optimizer step, not twice per micro-batch;
that is the fast mode whenever the 180 GB of a B200 hold them.

Overlap.  Gradient reduce-scatter of a unit starts on a side stream as soon as
that unit's backward finishes (a hook on the unit's inputs), only on the
micro-batch that syncs.  Parameter all-gathers of the next step are issued per
unit in forward order right after the optimizer step; each unit's forward
waits only for its own gather.

Resharding (``reshard_after_forward=True``, FSDP2's option of that name,
reference: mvp_engine/distributed/fsdp2.py:82-167).  Decoder units then keep only
this rank's bf16 slice (``wshard``) between uses; their full weights live in one
of two staging slots (units alternate) only while the unit runs, in forward and
again in backward.  Each unit's gather is issued one unit ahead on the comm
stream (the next unit in forward, the previous one in backward), after an event
that orders it behind the last kernel that read the slot, so it overlaps the
current unit's compute.  The gather is NCCL's all-gather (``comm="nccl"``) or the
engine's peer pull (``comm="fused"``): every rank reads the other ranks' slices
straight out of their symmetric shard buffers.  The root unit (embeddings, final
norm, LM head) stays resident.  Gradients accumulate in the full-size fp32 buffer
across micro-batches and are reduce-scattered on the syncing micro-batch, as
torch FSDP2 does when gradient sync is off between micro-batches.

Checkpoints.  ``checkpoint_state_dict`` returns HF-named tensors; on more than
one rank they are DTensors with ``Shard(0)`` placements over the shard mesh,
exactly the layout torch FSDP2 checkpoints with, rebuilt transiently from the
flat shards (one unit at a time, offloaded to CPU).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Any, Callable, Iterable, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from ..utils.log import logger

_ALIGN = 64  # elements; keeps every parameter view 128-byte aligned for TMA


@dataclass
class _Entry:
    fqns: list[str]  # all names that alias this parameter (tied weights)
    owners: list[tuple[nn.Module, str]]
    shape: torch.Size
    numel: int
    offset: int  # in the unit's full layout
    requires_grad: bool
    tp_partial: bool = False  # replicated over tensor parallelism, gradient summed over the tensor group
    tp_replicated: bool = False  # same value on every tensor rank (partial or not)
    tp_slice: Optional[tuple] = None  # (full shape, dim, start, stop): this rank's slice of a sharded weight

    @property
    def logical_shape(self) -> torch.Size:
        """Shape of the parameter as checkpoints store it (the full tensor for tensor-parallel slices)."""
        return torch.Size(self.tp_slice[0]) if self.tp_slice is not None else self.shape


@dataclass
class _PeerState:
    buf: torch.Tensor  # symmetric fp32 gradient buffer of all trainable units
    slots: torch.Tensor  # symmetric int64 signal slots [8]
    handles: tuple
    peer_bufs: list[int]
    peer_slots: list[int]
    my_slots: int
    offsets: dict[int, int]


@dataclass
class FlatUnit:
    index: int
    name: str
    module: Optional[nn.Module]
    entries: list[_Entry] = field(default_factory=list)
    total: int = 0
    padded: int = 0
    shard: int = 0
    trainable: bool = True
    full: Optional[torch.Tensor] = None
    grad: Optional[torch.Tensor] = None
    master: Optional[torch.Tensor] = None
    grad_shard: Optional[torch.Tensor] = None
    exp_avg: Optional[torch.Tensor] = None
    exp_avg_sq: Optional[torch.Tensor] = None
    ag_event: Optional[torch.cuda.Event] = None
    rs_event: Optional[torch.cuda.Event] = None
    rs_pending: bool = False
    views: dict[str, torch.Tensor] = field(default_factory=dict)
    resharded: bool = False  # full weights only while the unit runs (staging slot), else wshard
    slot: int = -1
    wshard: Optional[torch.Tensor] = None  # this rank's bf16 slice when resharded
    rep_end: int = 0  # entries [0, rep_end) are tensor-parallel partial (summed over the tensor group)
    repl_end: int = 0  # entries [0, repl_end) are replicated over the tensor group (partial or complete)

    def local_range(self, rank: int) -> tuple[int, int]:
        return rank * self.shard, (rank + 1) * self.shard

    def own_compute_slice(self, rank: int) -> torch.Tensor:
        """Where this rank's bf16 weights live between steps (the optimizer writes here)."""
        if self.resharded:
            return self.wshard
        lo, hi = self.local_range(rank)
        return self.full[lo:hi]


class _UnitBackwardHook(torch.autograd.Function):
    """Identity on the unit's inputs; its backward runs after every op of the unit."""

    @staticmethod
    def forward(ctx, owner, unit_index, *xs):
        ctx.owner = owner
        ctx.unit_index = unit_index
        return xs if len(xs) > 1 else xs[0]

    @staticmethod
    def backward(ctx, *grads):
        ctx.owner._on_unit_backward_done(ctx.unit_index)
        return (None, None) + grads


class _UnitBackwardStartHook(torch.autograd.Function):
    """Identity on the unit's outputs; its backward runs before any op of the unit's backward."""

    @staticmethod
    def forward(ctx, owner, unit_index, *xs):
        ctx.owner = owner
        ctx.unit_index = unit_index
        return xs if len(xs) > 1 else xs[0]

    @staticmethod
    def backward(ctx, *grads):
        ctx.owner._on_unit_backward_start(ctx.unit_index)
        return (None, None) + grads


def _dtype(d: Any) -> torch.dtype:
    if isinstance(d, torch.dtype):
        return d
    return {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32, "bf16": torch.bfloat16,
            "fp32": torch.float32}[str(d)]


class NativeFSDP(nn.Module):
    """Wrap ``model`` with flat-buffer sharded data parallelism over ``group``.

    Args:
        model: the module (parameters may be fp32 masters; they are copied).
        group: data-parallel process group (None -> single rank).
        device: compute device.
        param_dtype: dtype of compute weights (bf16 under mixed precision).
        unit_classes: class names that form their own unit (default: the
            model's ``_no_split_modules``).
        comm: ``"nccl"`` (torch.distributed collectives) or ``"fused"`` (the
            engine's own NVLink kernels where available).
    """

    def __init__(self, model: nn.Module, group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None, param_dtype: Any = torch.bfloat16,
                 unit_classes: Optional[Iterable[str]] = None, comm: str = "nccl",
                 shard_mesh: Any = None, tp_group: Optional[dist.ProcessGroup] = None,
                 reshard_after_forward: bool = False, replicate_group: Optional[dist.ProcessGroup] = None) -> None:
        super().__init__()
        # HSDP: parameters sharded over `group`, replicated over `replicate_group`, whose ranks average the
        # reduce-scattered gradient shards (reference: mvp_engine/distributed/parallel_mesh.py:144-164)
        self.replicate_group = replicate_group
        self.rep_world = (dist.get_world_size(replicate_group)
                          if (replicate_group is not None and dist.is_initialized()) else 1)
        self.reshard_after_forward = bool(reshard_after_forward)
        self._slots: list[torch.Tensor] = []
        self._slot_owner = [-1, -1]  # unit index whose full weights each staging slot holds (-1: none)
        self._phase = "forward"
        self._wpeer = None  # symmetric bf16 shard buffer for the peer-pull gather
        self._gather_job = None  # (unit index, ops.GatherJob) queued for the next large GEMM
        # Peer-pull gathers ride in the next large GEMM (MVP_FSDP_GATHER=gemm, default) or run as a
        # stand-alone kernel on the comm stream (=kernel); copy CTAs and the smallest carrying GEMM:
        self._gather_in_gemm = os.environ.get("MVP_FSDP_GATHER", "gemm") == "gemm"
        self._gather_ctas = int(os.environ.get("MVP_FSDP_GATHER_CTAS", "24"))
        # a GEMM carries the gather when it runs at least about as long as the remote bytes take over NVLink:
        # FLOPs >= remote bytes x 1500 (about 1.4 PFLOP/s over 0.9 of 770 GB/s, halved); MVP_FSDP_GATHER_MIN_MNK overrides the bound
        self._gather_flops_per_byte = 1500.0
        self._gather_min_mnk_env = os.environ.get("MVP_FSDP_GATHER_MIN_MNK")
        self.module = model
        self.group = group
        self.tp_group = tp_group
        self.tp_world = dist.get_world_size(tp_group) if (tp_group is not None and dist.is_initialized()) else 1
        self.world = dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1
        self.rank = dist.get_rank(group) if (group is not None and dist.is_initialized()) else 0
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        if self.device.type == "meta":
            raise ValueError("NativeFSDP needs a real device for its buffers (got meta)")
        self.param_dtype = _dtype(param_dtype)
        self.comm = comm
        self.shard_mesh = shard_mesh
        self._sync_grads = True
        # Gradients are averaged over the data-parallel ranks (FSDP2 / DDP semantics): the
        # reduce-scatter sums, and the 1/world factor rides in the optimizer's gradient scale.
        self._grad_scale = 1.0 / (self.world * self.rep_world)
        self._norm_sq: Optional[torch.Tensor] = None
        self._max_norm: Optional[float] = None
        cls_names = set(unit_classes) if unit_classes else set(getattr(model, "_no_split_modules", []) or [])
        self.units: list[FlatUnit] = []
        self._comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self._build_units(cls_names)
        # Shard masters are registered as parameters (their .grad is the fp32
        # gradient shard) so generic code -- model.parameters(), torch optimizers,
        # p.grad.mul_(...) -- works on the sharded state.
        self.shard_params = nn.ParameterList()
        for u in self.units:
            if u.trainable:
                p = nn.Parameter(u.master, requires_grad=True)
                u.master = p
                self.shard_params.append(p)
        self._attach_grads()
        self._install_hooks()
        self._gather_all(initial=True)

    # ----------------------------------------------------------- layout
    def _build_units(self, cls_names: set[str]) -> None:
        model = self.module
        unit_of_module: dict[int, int] = {}
        ordered: list[tuple[str, nn.Module]] = []
        for name, mod in model.named_modules():
            if type(mod).__name__ in cls_names and not any(name.startswith(p + ".") for p, _ in ordered):
                ordered.append((name, mod))
        # The root unit (index 0) gathers first: embeddings run before any block.
        self.units.append(FlatUnit(0, "<root>", None))
        for i, (name, mod) in enumerate(ordered):
            self.units.append(FlatUnit(i + 1, name, mod))
            unit_of_module[id(mod)] = i + 1

        def owning_unit(fqn: str) -> int:
            best, best_len = 0, -1
            for u in self.units[1:]:
                if (fqn == u.name or fqn.startswith(u.name + ".")) and len(u.name) > best_len:
                    best, best_len = u.index, len(u.name)
            return best

        seen: dict[int, _Entry] = {}
        for mod_name, mod in model.named_modules():
            for pname, p in list(mod._parameters.items()):
                if p is None:
                    continue
                fqn = f"{mod_name}.{pname}" if mod_name else pname
                if id(p) in seen:
                    seen[id(p)].fqns.append(fqn)
                    seen[id(p)].owners.append((mod, pname))
                    continue
                unit = self.units[owning_unit(fqn)]
                e = _Entry([fqn], [(mod, pname)], p.shape, p.numel(), 0, p.requires_grad,
                           tp_partial=self.tp_world > 1 and bool(getattr(p, "_mvp_tp_partial", False)),
                           tp_replicated=self.tp_world > 1 and not getattr(p, "_mvp_tp_sharded", False),
                           tp_slice=getattr(p, "_mvp_tp_slice", None) if self.tp_world > 1 else None)
                seen[id(p)] = e
                unit.entries.append(e)
        # Frozen parameters of a unit move to a sibling unit without optimizer state.
        extra: list[FlatUnit] = []
        for u in self.units:
            frozen = [e for e in u.entries if not e.requires_grad]
            if frozen and len(frozen) < len(u.entries):
                u.entries = [e for e in u.entries if e.requires_grad]
                extra.append(FlatUnit(-1, u.name + "<frozen>", u.module, frozen, trainable=False))
            elif frozen:
                u.trainable = False
        for x in extra:
            x.index = len(self.units)
            self.units.append(x)
        params = {id(p): p for p in model.parameters()}
        by_entry = {id(e): params_id for params_id, e in seen.items()}
        for u in self.units:
            off = 0
            # tensor-partial entries first, then other tensor-replicated ones, then tensor shards
            u.entries.sort(key=lambda e: (not e.tp_partial, not e.tp_replicated))
            for e in u.entries:
                e.offset = off
                off += int(math.ceil(e.numel / _ALIGN) * _ALIGN)
                if e.tp_partial:
                    u.rep_end = off
                if e.tp_replicated:
                    u.repl_end = off
            u.total = off
            quantum = _ALIGN * self.world
            u.padded = max(quantum, int(math.ceil(off / quantum) * quantum))
            u.shard = u.padded // self.world
        self._peer = self._setup_peer_collectives()
        self._plan_resharding()
        for u in self.units:
            self._materialise(u, {id(e): params[by_entry[id(e)]] for e in u.entries})

    def _setup_peer_collectives(self) -> Optional["_PeerState"]:
        """Gradient buffers in one symmetric (peer-mapped) allocation for the pull reduce-scatter kernel.

        Used for ``comm="fused"`` on CUDA with 2..8 data-parallel ranks; anything else (or a setup
        failure, reported once) keeps NCCL's reduce-scatter.
        """
        if self.comm != "fused" or self.world <= 1 or self.device.type != "cuda" or self.world > 8:
            return None
        if os.environ.get("MVP_FUSED_COMM", "1") == "0":
            return None
        try:
            import torch.distributed._symmetric_memory as symm

            try:
                if symm.get_backend(self.device) != "CUDA":
                    symm.set_backend("CUDA")
            except Exception:  # noqa: BLE001 - older / newer APIs: keep the default backend
                pass
            group = self.group if self.group is not None else dist.group.WORLD
            try:
                symm.enable_symm_mem_for_group(group.group_name)
            except Exception:  # noqa: BLE001 - not needed (or not present) on newer torch
                pass
            total = sum(u.padded for u in self.units if u.trainable)
            buf = symm.empty(max(total, 4), dtype=torch.float32, device=self.device)
            buf.zero_()
            slots = symm.empty(8, dtype=torch.int64, device=self.device)
            slots.zero_()
            torch.cuda.synchronize(self.device)
            h_buf = symm.rendezvous(buf, group)
            h_slots = symm.rendezvous(slots, group)
            h_slots.barrier()
            off, offsets = 0, {}
            for u in self.units:
                if u.trainable:
                    offsets[u.index] = off
                    off += u.padded
            return _PeerState(buf=buf, slots=slots, handles=(h_buf, h_slots),
                              peer_bufs=[int(x) for x in h_buf.buffer_ptrs],
                              peer_slots=[int(x) for x in h_slots.buffer_ptrs],
                              my_slots=int(slots.data_ptr()), offsets=offsets)
        except Exception as exc:  # noqa: BLE001 - fall back to NCCL, loudly
            from ..utils.log import simple_info

            simple_info(f"native FSDP: peer-memory reduce-scatter unavailable ({type(exc).__name__}: {exc}); "
                        "using NCCL reduce-scatter", level="warning")
            return None

    def _plan_resharding(self) -> None:
        """Pick the resharded units (trainable decoder blocks), give each a staging slot (alternating in
        forward order) and its bf16 shard; allocate two slots of the largest such unit."""
        if not self.reshard_after_forward or self.world == 1:
            return
        chosen = [u for u in self.units if u.module is not None and u.trainable and "<frozen>" not in u.name]
        if len(chosen) < 2:
            return
        for k, u in enumerate(chosen):
            u.resharded, u.slot = True, k % 2
        biggest = max(u.padded for u in chosen)
        self._slots = [torch.zeros(biggest, dtype=self.param_dtype, device=self.device) for _ in range(2)]
        total = sum(u.shard for u in chosen)
        self._wshard_base = self._alloc_weight_shards(total)
        off = 0
        self._wshard_off: dict[int, int] = {}
        for u in chosen:
            u.wshard = self._wshard_base[off:off + u.shard]
            self._wshard_off[u.index] = off
            off += u.shard

    def _alloc_weight_shards(self, total: int) -> torch.Tensor:
        """bf16 shard storage of the resharded units: symmetric (peer-readable) memory for the pull gather."""
        if self.comm == "fused" and self.device.type == "cuda" and 1 < self.world <= 8 and \
                os.environ.get("MVP_FUSED_COMM", "1") != "0":
            try:
                import torch.distributed._symmetric_memory as symm

                group = self.group if self.group is not None else dist.group.WORLD
                buf = symm.empty(max(total, 8), dtype=self.param_dtype, device=self.device)
                buf.zero_()
                flags = symm.empty(8, dtype=torch.int64, device=self.device)
                flags.zero_()
                torch.cuda.synchronize(self.device)
                h_buf = symm.rendezvous(buf, group)
                h_flags = symm.rendezvous(flags, group)
                h_flags.barrier()
                self._wpeer = dict(buf=buf, flags=flags, handles=(h_buf, h_flags),
                                   bufs=[int(x) for x in h_buf.buffer_ptrs],
                                   flag_ptrs=[int(x) for x in h_flags.buffer_ptrs], epoch=0)
                return buf[:total]
            except Exception as exc:  # noqa: BLE001 - fall back to NCCL all-gathers, loudly
                from ..utils.log import simple_info

                simple_info(f"native FSDP: peer-pull parameter gather unavailable ({type(exc).__name__}: {exc}); "
                            "using NCCL all-gather", level="warning")
                self._wpeer = None
        return torch.zeros(total, dtype=self.param_dtype, device=self.device)

    def _next_seq(self) -> int:
        self._seq = getattr(self, "_seq", 0) + 1
        return self._seq

    def _materialise(self, u: FlatUnit, src: dict[int, torch.Tensor]) -> None:
        dev = self.device
        if u.resharded:
            u.full = self._slots[u.slot][:u.padded]
            u.full.zero_()
        else:
            u.full = torch.zeros(u.padded, dtype=self.param_dtype, device=dev)
        lo, hi = u.local_range(self.rank)
        if u.trainable:
            u.master = torch.zeros(u.shard, dtype=torch.float32, device=dev)
        init = getattr(self.module, "init_param_", None)
        seed = getattr(self.module, "_init_seed", None)
        with torch.no_grad():
            for e in u.entries:
                p = src[id(e)]
                if p.is_meta:
                    # Materialise straight into the flat buffers, one parameter at a time.
                    if init is None:
                        raise RuntimeError(f"{e.fqns[0]} is on the meta device and the model has no init_param_")
                    cut = getattr(p, "_mvp_tp_slice", None)  # a tensor-parallel slice of a larger weight
                    if cut is None:
                        tmp = torch.empty(e.shape, dtype=torch.float32, device=dev)
                        init(e.fqns[0], tmp, seed)
                    else:
                        full_shape, dim, start, stop = cut
                        tmp = torch.empty(full_shape, dtype=torch.float32, device=dev)
                        init(e.fqns[0], tmp, seed)
                        tmp = tmp.narrow(dim, start, stop - start).contiguous()
                    flat = tmp.reshape(-1)
                else:
                    flat = p.detach().reshape(-1)
                u.full[e.offset:e.offset + e.numel].copy_(flat)
                if u.trainable:
                    a, b = max(lo, e.offset), min(hi, e.offset + e.numel)
                    if a < b:
                        u.master[a - lo:b - lo].copy_(flat[a - e.offset:b - e.offset].float())
        if u.trainable:
            if self._peer is not None:
                o = self._peer.offsets[u.index]
                u.grad = self._peer.buf[o:o + u.padded]
            else:
                u.grad = torch.zeros(u.padded, dtype=torch.float32, device=dev)
            u.grad_shard = u.grad if self.world == 1 else torch.zeros(u.shard, dtype=torch.float32, device=dev)
            u.exp_avg = torch.zeros_like(u.master)
            u.exp_avg_sq = torch.zeros_like(u.master)
        for e in u.entries:
            view = u.full[e.offset:e.offset + e.numel].view(e.shape)
            if u.trainable:
                gview = u.grad[e.offset:e.offset + e.numel].view(e.shape)
                # Native kernels accumulate weight gradients straight into the flat fp32 buffer
                # (and give autograd none); any other op (eager PyTorch: biases, LayerNorm, ...) lets
                # autograd produce .grad, which the hook folds into the same buffer.
                view._mvp_grad_acc = gview
                view.requires_grad_(True)
                view.register_post_accumulate_grad_hook(_make_fold_hook(gview))
            for mod, pname in e.owners:
                del mod._parameters[pname]
                setattr(mod, pname, view)
            u.views[e.fqns[0]] = view
        if u.module is not None:
            self._publish_fused(u)
        if u.resharded:  # keep this rank's slice; the slot is shared with every other unit of its parity
            with torch.no_grad():
                u.wshard.copy_(u.full[lo:hi])
            self._slot_owner[u.slot] = u.index

    def _publish_fused(self, u: FlatUnit) -> None:
        """Expose contiguous q/k/v and gate/up as single GEMM operands when laid out back to back."""
        mod = u.module
        if not hasattr(mod, "_fused"):
            return
        fused: dict[str, torch.Tensor] = {}
        for key, names in (("qkv", ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight")),
                           ("gate_up", ("mlp.gate_proj.weight", "mlp.up_proj.weight"))):
            full_names = [f"{u.name}.{n}" for n in names]
            ents = [next((e for e in u.entries if e.fqns[0] == fn), None) for fn in full_names]
            if any(e is None for e in ents):
                continue
            contiguous = all(ents[i].offset + ents[i].numel == ents[i + 1].offset for i in range(len(ents) - 1))
            if not contiguous or len({e.shape[1] for e in ents}) != 1:
                continue
            rows = sum(e.shape[0] for e in ents)
            view = u.full[ents[0].offset:ents[0].offset + rows * ents[0].shape[1]].view(rows, ents[0].shape[1])
            if u.trainable:
                view._mvp_grad_acc = u.grad[ents[0].offset:ents[0].offset + view.numel()].view(view.shape)
            fused[key] = view
        mod._fused = fused or None

    # ------------------------------------------------------------ hooks
    def _install_hooks(self) -> None:
        self._resharded_order = [u.index for u in self.units if u.resharded]
        for u in self.units[1:]:
            if u.module is None or "<frozen>" in u.name:
                continue
            u.module.register_forward_pre_hook(self._make_pre_hook(u.index), with_kwargs=False)
            if u.resharded:
                u.module.register_forward_hook(self._make_post_hook(u.index))

    def _make_post_hook(self, idx: int) -> Callable:
        """Wrap a resharded unit's outputs so its backward first brings the unit's weights back."""

        def hook(module, args, output):
            if not torch.is_grad_enabled() or not self.module.training:
                return None
            outs = output if isinstance(output, tuple) else (output,)
            live = [o for o in outs if isinstance(o, torch.Tensor) and o.requires_grad]
            if not live:
                return None
            wrapped = _UnitBackwardStartHook.apply(self, idx, *live)
            wrapped = wrapped if isinstance(wrapped, tuple) else (wrapped,)
            it = iter(wrapped)
            res = tuple(next(it) if (isinstance(o, torch.Tensor) and o.requires_grad) else o for o in outs)
            return res if isinstance(output, tuple) else res[0]

        return hook

    def _neighbour(self, idx: int, step: int) -> Optional[int]:
        order = self._resharded_order
        k = order.index(idx) + step
        return order[k] if 0 <= k < len(order) else None

    def _on_unit_backward_start(self, idx: int) -> None:
        self._phase = "backward"
        self._ensure_gathered(idx)
        self._wait_gather(idx)
        prev = self._neighbour(idx, -1)
        if prev is not None:
            self._ensure_gathered(prev)  # prefetch: overlaps this unit's backward

    def _make_pre_hook(self, idx: int) -> Callable:
        def hook(module, args):
            if self.units[idx].resharded:
                self._ensure_gathered(idx)
            self._wait_gather(idx)
            for sib in self._siblings(idx):
                self._wait_gather(sib)
            if self.units[idx].resharded and self._phase == "forward":
                nxt = self._neighbour(idx, +1)
                if nxt is not None:
                    self._ensure_gathered(nxt)  # prefetch: overlaps this unit's forward
            if not torch.is_grad_enabled() or not self.module.training:
                return None
            tensors = [a for a in args if isinstance(a, torch.Tensor) and a.requires_grad]
            if not tensors:
                return None
            hooked = _UnitBackwardHook.apply(self, idx, *tensors)
            hooked = hooked if isinstance(hooked, tuple) else (hooked,)
            it = iter(hooked)
            return tuple(next(it) if (isinstance(a, torch.Tensor) and a.requires_grad) else a for a in args)

        return hook

    def _siblings(self, idx: int) -> list[int]:
        name = self.units[idx].name
        return [u.index for u in self.units if u.name == name + "<frozen>"]

    def _on_unit_backward_done(self, idx: int) -> None:
        if self._sync_grads:
            self._reduce_scatter(idx)

    # --------------------------------------------------- collectives
    def _wait_gather(self, idx: int) -> None:
        if self.units[idx].resharded:
            self._flush_gather_job(idx)
        ev = self.units[idx].ag_event
        if ev is not None and self.device.type == "cuda":
            torch.cuda.current_stream(self.device).wait_event(ev)
            self.units[idx].ag_event = None

    def _ensure_gathered(self, idx: int) -> None:
        """Issue the gather of resharded unit ``idx`` into its slot unless the slot already holds it."""
        u = self.units[idx]
        if self._slot_owner[u.slot] == idx:
            return
        self._slot_owner[u.slot] = idx
        self._gather(u)

    def _gather(self, u: FlatUnit) -> None:
        if self.world == 1:
            return
        if u.resharded:
            self._gather_resharded(u)
            return
        lo, hi = u.local_range(self.rank)
        if self._comm_stream is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._comm_stream.wait_event(ev)
            with torch.cuda.stream(self._comm_stream):
                dist.all_gather_into_tensor(u.full, u.full[lo:hi], group=self.group)
                u.ag_event = torch.cuda.Event()
                u.ag_event.record(self._comm_stream)
                u.full.record_stream(self._comm_stream)
        else:
            parts = [torch.empty(u.shard, dtype=u.full.dtype) for _ in range(self.world)]
            dist.all_gather(parts, u.full[lo:hi].detach().clone(), group=self.group)
            with torch.no_grad():
                u.full.copy_(torch.cat(parts))

    def _gather_resharded(self, u: FlatUnit) -> None:
        """Full weights of ``u`` into its staging slot from every rank's bf16 shard.

        On the comm stream, behind an event of the compute stream: every kernel issued so far (the last
        reader of this slot among them) is ordered before the copy; the unit's own ops wait for
        ``u.ag_event``."""
        cur = torch.cuda.current_stream(self.device) if self._comm_stream is not None else None
        # Saved tensors of the unit's earlier use (forward, for its backward) are views of this slot: the
        # refill restores exactly those values, so the slot's version counter is kept as it was.
        keep_version = torch.autograd._unsafe_preserve_version_counter(self._slots[u.slot])
        if cur is None:  # CPU / gloo: synchronous
            parts = [torch.empty(u.shard, dtype=u.full.dtype) for _ in range(self.world)]
            dist.all_gather(parts, u.wshard.detach().clone(), group=self.group)
            with torch.no_grad(), keep_version:
                u.full.copy_(torch.cat(parts))
            return
        if self._wpeer is not None and self._gather_in_gemm:
            # Fused path: the pull rides in extra CTAs of the next large GEMM on the compute stream (the
            # current unit's), which comes after every earlier reader of the slot and before every use
            # of the gathered unit.  A job no GEMM took is flushed by _wait_gather.
            from .. import ops as _ops

            self._flush_gather_job()
            wp = self._wpeer
            remote = (self.world - 1) * u.shard * u.full.element_size()
            min_flops = (int(self._gather_min_mnk_env) if self._gather_min_mnk_env is not None
                         else int(remote * self._gather_flops_per_byte))
            job = _ops.GatherJob(wp["bufs"], wp["flag_ptrs"], self._wshard_off[u.index], u.shard, wp["epoch"],
                                 u.full, self._gather_ctas, min_flops)
            self._gather_job = (u.index, job)
            u.ag_event = None
            _ops.set_pending_gather(job)
            return
        ev = torch.cuda.Event()
        ev.record(cur)
        self._comm_stream.wait_event(ev)
        with torch.cuda.stream(self._comm_stream), torch.no_grad(), keep_version:
            if self._wpeer is not None:
                from .. import ops as _ops

                wp = self._wpeer
                off = self._wshard_off[u.index]
                _ops.peer_gather_shards(wp["bufs"], wp["flag_ptrs"], self.rank, off, u.shard, wp["epoch"], u.full)
            else:
                dist.all_gather_into_tensor(u.full, u.wshard, group=self.group)
            u.ag_event = torch.cuda.Event()
            u.ag_event.record(self._comm_stream)

    def _flush_gather_job(self, idx: Optional[int] = None) -> None:
        """Launch a queued GEMM-carried gather that no GEMM took (all of them, or only unit ``idx``'s) as the
        stand-alone pull kernel on the compute stream, ahead of the gathered unit's first use."""
        pending = getattr(self, "_gather_job", None)
        if pending is None or (idx is not None and pending[0] != idx):
            return
        from .. import ops as _ops

        unit_idx, job = pending
        self._gather_job = None
        if _ops.pending_gather() is job:
            _ops.set_pending_gather(None)
        if job.consumed:
            return
        bufs, flags, off, shard, epoch = job.args
        with torch.no_grad(), torch.autograd._unsafe_preserve_version_counter(self._slots[self.units[unit_idx].slot]):
            _ops.peer_gather_shards(bufs, flags, self.rank, off, shard, epoch, job.slot)

    @torch.no_grad()
    def _gather_all(self, initial: bool = False) -> None:
        for u in self.units:
            if initial and self.world > 1 and u.trainable:
                # masters were copied from the full init; refresh this rank's slice
                u.own_compute_slice(self.rank).copy_(u.master.detach())
            if u.resharded:
                continue  # gathered on first use
            self._gather(u)
        if self._slots:
            self._slot_owner = [-1, -1]
            self._publish_weight_epoch()

    def _publish_weight_epoch(self) -> None:
        """Tell the peers that this rank's bf16 shards are final for the coming step (peer-pull gather)."""
        if self._wpeer is None:
            return
        from .. import ops as _ops

        wp = self._wpeer
        wp["epoch"] += 1
        _ops.publish_epoch(int(wp["flags"].data_ptr()), wp["epoch"])

    def _reduce_scatter(self, idx: int) -> None:
        u = self.units[idx]
        if not u.trainable or u.rs_pending:
            return
        u.rs_pending = True
        tp_sum = self.tp_world > 1 and u.rep_end > 0
        if self.world == 1 and not tp_sum:
            return
        if self._comm_stream is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._comm_stream.wait_event(ev)
            with torch.cuda.stream(self._comm_stream):
                if tp_sum:
                    dist.all_reduce(u.grad[:u.rep_end], group=self.tp_group)
                if self.world > 1 and self._peer is not None:
                    from .. import ops as _ops

                    pe = self._peer
                    _ops.peer_reduce_scatter(pe.peer_bufs, pe.peer_slots, pe.my_slots, self.rank,
                                             pe.offsets[u.index], u.shard, self._next_seq(), u.grad_shard)
                elif self.world > 1:
                    dist.reduce_scatter_tensor(u.grad_shard, u.grad, op=dist.ReduceOp.SUM, group=self.group)
                if self.rep_world > 1 and self.world > 1:
                    dist.all_reduce(u.grad_shard, group=self.replicate_group)
                u.rs_event = torch.cuda.Event()
                u.rs_event.record(self._comm_stream)
        else:
            if tp_sum:
                part = u.grad[:u.rep_end].detach().clone()
                dist.all_reduce(part, group=self.tp_group)
                with torch.no_grad():
                    u.grad[:u.rep_end].copy_(part)
            if self.world == 1:
                return
            buf = u.grad.detach().clone()
            dist.all_reduce(buf, group=self.group)
            lo, hi = u.local_range(self.rank)
            part = buf[lo:hi].clone()
            if self.rep_world > 1:
                dist.all_reduce(part, group=self.replicate_group)
            with torch.no_grad():
                u.grad_shard.copy_(part)

    def finish_grad_sync(self) -> None:
        """Reduce-scatter units whose hook did not fire (root, embeddings) and wait for all."""
        for u in reversed(self.units):
            if u.trainable and not u.rs_pending:
                self._reduce_scatter(u.index)
        cur = torch.cuda.current_stream(self.device) if self.device.type == "cuda" else None
        for u in self.units:
            if u.rs_event is not None and cur is not None:
                cur.wait_event(u.rs_event)
                u.rs_event = None

    # --------------------------------------------------------- API
    def set_requires_gradient_sync(self, requires_gradient_sync: bool, *, recurse: bool = True) -> None:
        self._sync_grads = bool(requires_gradient_sync)

    def forward(self, *args, **kwargs):
        self._phase = "forward"
        self._wait_gather(0)
        for sib in self._siblings(0):
            self._wait_gather(sib)
        if self.module.training and torch.is_grad_enabled() and self.device.type == "cuda":
            # Give the embedding backward a tensor that requires grad, so it runs even
            # though the weight view itself does not require grad.
            for mod in self._embed_owners():
                mod._embed_anchor = self._anchor
        return self.module(*args, **kwargs)

    def _embed_owners(self) -> list[nn.Module]:
        owners = getattr(self, "_embed_owner_cache", None)
        if owners is None:
            owners = [m for m in self.module.modules() if hasattr(m, "embed_tokens")]
            self._embed_owner_cache = owners
        return owners

    @property
    def _anchor(self) -> torch.Tensor:
        a = getattr(self, "_anchor_t", None)
        if a is None:
            a = torch.zeros((), device=self.device, requires_grad=True)
            self._anchor_t = a
        return a

    def grad_shards(self) -> list[torch.Tensor]:
        return [u.grad_shard for u in self.units if u.trainable]

    def scale_gradients_(self, factor: float) -> None:
        """Fold a gradient multiplier (token normalisation) into the next optimizer update."""
        self._grad_scale *= float(factor)

    @torch.no_grad()
    def clip_grad_norm_(self, max_norm: float, norm_type: float = 2.0) -> torch.Tensor:
        """Global norm of (scaled) gradients; the clip itself is folded into the optimizer update."""
        if norm_type != 2.0:
            raise NotImplementedError("native FSDP clips with the 2-norm")
        self.finish_grad_sync()
        from .. import ops

        parts = [ops.sumsq(g) for g in self.grad_shards()]
        nsq = torch.stack(parts).sum().reshape(1) if parts else torch.zeros(1, device=self.device)
        if self.tp_world > 1:
            # Replicated ranges are identical on every tensor rank (partial ones after their
            # all-reduce): count them once in the sum over the tensor group.
            rep = [ops.sumsq(u.grad_shard[:max(0, min(u.repl_end, hi) - lo)]) for u in self.units
                   if u.trainable and u.repl_end > 0 for lo, hi in [u.local_range(self.rank)] if u.repl_end > lo]
            if rep:
                nsq = nsq - torch.stack(rep).sum().reshape(1) * (1.0 - 1.0 / self.tp_world)
            dist.all_reduce(nsq, group=self.tp_group)
        if self.world > 1:
            dist.all_reduce(nsq, group=self.group)
        self._norm_sq = nsq
        self._max_norm = float(max_norm)
        return nsq.sqrt()[0] * self._grad_scale

    def _attach_grads(self) -> None:
        for u in self.units:
            if u.trainable:
                u.master.grad = u.grad_shard[: u.shard] if u.grad_shard is u.grad else u.grad_shard

    def attach_optimizer(self, optimizer: torch.optim.Optimizer) -> torch.optim.Optimizer:
        """For a stock torch optimizer over ``shard_params``: after each ``step`` refresh the
        compute weights from the updated masters and start the next all-gathers."""

        def post(opt, args, kwargs):
            with torch.no_grad():
                for u in self.units:
                    if u.trainable:
                        u.own_compute_slice(self.rank).copy_(u.master.detach())
            self.after_optimizer_step()

        if not getattr(optimizer, "_mvp_native_step", False):
            optimizer.register_step_pre_hook(lambda opt, a, k: self.finish_grad_sync())
            optimizer.register_step_post_hook(post)
        return optimizer

    def after_optimizer_step(self) -> None:
        """Zero gradient buffers, reset per-step state and start next step's all-gathers."""
        if self._peer is not None:
            # peers may still be pulling from this rank's gradient buffers: meet them first
            from .. import ops as _ops

            pe = self._peer
            _ops.peer_barrier(pe.peer_slots, pe.my_slots, self.rank, self._next_seq())
        for u in self.units:
            if u.trainable:
                u.grad.zero_()
                if u.grad_shard is not u.grad:
                    u.grad_shard.zero_()
            u.rs_pending = False
        self._grad_scale = 1.0 / (self.world * self.rep_world)
        self._norm_sq = None
        self._max_norm = None
        self._attach_grads()
        for u in self.units:
            if u.trainable and not u.resharded:
                self._gather(u)
        if self._slots:  # the slots hold last step's weights: every resharded unit gathers again
            self._slot_owner = [-1, -1]
            self._publish_weight_epoch()

    def logical_parameter_counts(self) -> tuple[int, int]:
        total = sum(e.numel for u in self.units for e in u.entries)
        trainable = sum(e.numel for u in self.units if u.trainable for e in u.entries)
        return total, trainable

    # ---------------------------------------------------- checkpoints
    def _shard_rows(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's Shard(0) chunk of a full tensor (torch.chunk semantics, as DTensor uses)."""
        chunks = torch.chunk(full, self.world, dim=0)
        return chunks[self.rank] if self.rank < len(chunks) else full.new_zeros((0,) + tuple(full.shape[1:]))

    def _to_dtensor(self, local: torch.Tensor, shape: torch.Size):
        from torch.distributed.tensor import DTensor, Replicate, Shard

        # HSDP: a 2-D (replicate, shard) mesh, FSDP2's placements for it
        placements = [Replicate(), Shard(0)] if self.shard_mesh.ndim == 2 else [Shard(0)]
        return DTensor.from_local(local, self.shard_mesh, placements, run_check=False, shape=shape,
                                  stride=torch.empty(shape, device="meta").stride())

    @torch.no_grad()
    def _full_fp32(self, u: FlatUnit, flat_shard: torch.Tensor) -> torch.Tensor:
        flat_shard = flat_shard.detach()
        if self.world == 1:
            return flat_shard
        if flat_shard.is_cuda:
            out = torch.empty(u.padded, dtype=flat_shard.dtype, device=flat_shard.device)
            dist.all_gather_into_tensor(out, flat_shard.contiguous(), group=self.group)
            return out
        parts = [torch.empty_like(flat_shard) for _ in range(self.world)]
        dist.all_gather(parts, flat_shard.contiguous(), group=self.group)
        return torch.cat(parts)

    @torch.no_grad()
    def _tp_full(self, e: _Entry, t: torch.Tensor) -> torch.Tensor:
        """The full logical tensor of a tensor-parallel slice: the tensor ranks' equal slices, in rank
        order, concatenated along the sharded dimension (every tensor rank calls this in the same order)."""
        if e.tp_slice is None:
            return t
        parts = [torch.empty_like(t) for _ in range(self.tp_world)]
        dist.all_gather(parts, t.contiguous(), group=self.tp_group)
        return torch.cat(parts, dim=e.tp_slice[1])

    def _iter_tensors(self, which: str, full: bool):
        for u in self.units:
            if which != "param" and not u.trainable:
                continue
            if which == "param":
                src = self._full_fp32(u, u.master) if u.trainable else u.full.float()
            else:
                src = self._full_fp32(u, getattr(u, which))
            for e in u.entries:
                t = self._tp_full(e, src[e.offset:e.offset + e.numel].view(e.shape))
                if full or self.world == 1:
                    yield e, t.detach().to("cpu", copy=True)
                else:
                    yield e, self._to_dtensor(self._shard_rows(t).detach().clone().cpu(), e.logical_shape)

    def _local_value(self, e: _Entry, v: Any) -> torch.Tensor:
        """A checkpoint value (full logical tensor or DTensor) as this rank's entry: cut to the tensor
        rank's slice for tensor-parallel weights."""
        t = self._full_from_value(v, e.logical_shape)
        if e.tp_slice is not None:
            _, dim, start, stop = e.tp_slice
            t = t.narrow(dim, start, stop - start)
        return t.reshape(-1)

    @torch.no_grad()
    def checkpoint_state_dict(self, full: bool = False) -> dict[str, Any]:
        out: dict[str, Any] = {}
        for e, t in self._iter_tensors("param", full):
            for fqn in e.fqns:
                out[fqn] = t
        return out

    @torch.no_grad()
    def load_checkpoint_state_dict(self, sd: dict[str, Any], full: bool = False) -> None:
        for u in self.units:
            stage = torch.zeros(u.padded, dtype=torch.float32, device=self.device)
            for e in u.entries:
                key = next((f for f in e.fqns if f in sd), None)
                if key is None:
                    continue
                stage[e.offset:e.offset + e.numel].copy_(self._local_value(e, sd[key]))
            lo, hi = u.local_range(self.rank)
            if u.trainable:
                u.master.copy_(stage[lo:hi])
            if u.resharded:
                u.wshard.copy_(stage[lo:hi].to(u.wshard.dtype))
            else:
                u.full.copy_(stage.to(u.full.dtype))
        if self._slots:
            self._slot_owner = [-1, -1]
            self._publish_weight_epoch()

    def _full_from_value(self, v: Any, shape: torch.Size) -> torch.Tensor:
        try:
            from torch.distributed.tensor import DTensor

            if isinstance(v, DTensor):
                v = v.full_tensor()
        except ImportError:  # pragma: no cover
            pass
        return v.to(self.device, torch.float32).reshape(shape)

    def optimizer_state_views(self, full: bool = False):
        """(fqns, step-independent tensors) for exp_avg / exp_avg_sq in checkpoint layout."""
        avg = list(self._iter_tensors("exp_avg", full))
        sq = list(self._iter_tensors("exp_avg_sq", full))
        return [(e.fqns, a, s) for (e, a), (_, s) in zip(avg, sq)]

    @torch.no_grad()
    def load_optimizer_views(self, state: dict[str, dict[str, Any]]) -> None:
        for u in self.units:
            if not u.trainable:
                continue
            for name in ("exp_avg", "exp_avg_sq"):
                stage = torch.zeros(u.padded, dtype=torch.float32, device=self.device)
                for e in u.entries:
                    key = next((f for f in e.fqns if f in state and name in state[f]), None)
                    if key is not None:
                        stage[e.offset:e.offset + e.numel].copy_(self._local_value(e, state[key][name]))
                lo, hi = u.local_range(self.rank)
                getattr(u, name).copy_(stage[lo:hi])


def _make_fold_hook(gview: torch.Tensor) -> Callable:
    def hook(t: torch.Tensor) -> None:
        if t.grad is not None:
            gview.add_(t.grad.to(gview.dtype))
            t.grad = None

    return hook
