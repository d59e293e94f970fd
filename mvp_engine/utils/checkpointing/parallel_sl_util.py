"""Checkpoint save / load with the reference's on-disk layout
(reference: mvp_engine/utils/checkpointing/parallel_sl_util.py:224-440)::

    <run>/checkpoints/iter_<step>/
        engine/rank_<r>.pt       per-rank RNG state (torch, python, numpy, cuda)
        model/ , optimizer/      torch.distributed.checkpoint (sharded backends)
        model.pt, optimizer.pt   rank-0 torch.save (DDP / unsharded backends)
        engine.pt                step, epoch, _accumulate_step, scheduler, scaler
        hf_model/model.safetensors  optional full HF-named export

The backend is inferred from the mesh like the reference does (``shard`` or
``tensor`` > 1 -> sharded DCP).  Model keys are the HF parameter names under
the ``"model"`` entry; optimizer state uses ``state.<fqn>.{step,exp_avg,
exp_avg_sq}`` plus ``param_groups`` -- the layout torch's
``get_optimizer_state_dict`` produces for FSDP2, so a checkpoint written by the
engine's native data-parallel runtime and one written by torch FSDP2 are
interchangeable.  Models that expose ``checkpoint_state_dict`` /
``load_checkpoint_state_dict`` (the native runtime) provide their own sharded
views; everything else goes through torch's state-dict helpers.
"""

from __future__ import annotations

import gc
import os
import random
from pathlib import Path
from typing import Any, Optional

import numpy as np
import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch import nn

from ...distributed.utils import get_rank, is_main_process
from ..log import simple_info

OPTIM_STATE_KEY = "state"
HF_MODEL_DIRNAME = "hf_model"


def _base(model: nn.Module) -> nn.Module:
    return getattr(model, "_orig_mod", model)


def _pg():
    return dist.group.WORLD if dist.is_available() and dist.is_initialized() else None


def _barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def infer_checkpoint_backend(mesh) -> str:
    if mesh is None:
        return "ddp"
    names = mesh.mesh_dim_names or ()
    for dim in ("shard", "tensor", "context"):
        if dim in names and mesh[dim].size() > 1:
            return "fsdp2"
    shape = tuple(mesh.shape)
    if len(shape) > 1 and any(s > 1 for s in shape[1:]) and not names:
        return "fsdp2"
    return "ddp"


def _is_native(model: nn.Module) -> bool:
    return hasattr(_base(model), "checkpoint_state_dict")


# ------------------------------------------------------------- state dicts
def model_state_dict(model: nn.Module, *, full: bool) -> dict[str, Any]:
    base = _base(model)
    if _is_native(base):
        return base.checkpoint_state_dict(full=full)
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    if hasattr(base, "module") and not full:
        return base.module.state_dict()
    return get_model_state_dict(base, options=StateDictOptions(full_state_dict=full, cpu_offload=True))


def optimizer_state_dict(model: nn.Module, optimizer, *, full: bool = False) -> dict[str, Any]:
    base = _base(model)
    if hasattr(optimizer, "checkpoint_state_dict"):
        return optimizer.checkpoint_state_dict(full=full)
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_optimizer_state_dict

    sd = get_optimizer_state_dict(base, optimizer, options=StateDictOptions(full_state_dict=full, cpu_offload=True))
    _fill_missing_optimizer_states(base, sd)
    return sd


def _fill_missing_optimizer_states(model: nn.Module, optim_sd: dict[str, Any]) -> int:
    """Trainable params with no optimizer state yet (never stepped) get an empty entry,
    so the DCP key set is stable from the first save (reference :99-114)."""
    state = optim_sd.get(OPTIM_STATE_KEY)
    if not isinstance(state, dict):
        return 0
    missing = 0
    for fqn, p in model.named_parameters():
        if p.requires_grad and fqn not in state and fqn.replace("_orig_mod.", "") not in state:
            state[fqn] = {}
            missing += 1
    return missing


def _rng_state() -> dict[str, Any]:
    st = {"torch_rng_state": torch.get_rng_state(), "python_rng_state": random.getstate(),
          "numpy_rng_state": np.random.get_state()}
    if torch.cuda.is_available():
        st["accelerator_type"] = "cuda"
        st["accelerator_rng_state"] = torch.cuda.get_rng_state()
    return st


def _restore_rng(st: dict[str, Any]) -> None:
    if "torch_rng_state" in st:
        torch.set_rng_state(st["torch_rng_state"])
    acc = st.get("accelerator_rng_state", st.get("cuda_rng_state"))
    if acc is not None and torch.cuda.is_available():
        torch.cuda.set_rng_state(acc)
    if "python_rng_state" in st:
        random.setstate(st["python_rng_state"])
    if "numpy_rng_state" in st:
        np.random.set_state(st["numpy_rng_state"])


# -------------------------------------------------------------------- save
def save_checkpoint(mesh, cur_checkpoint_dir: Path, model: nn.Module, optimizer=None, scheduler=None, scaler=None,
                    step: int = 0, epoch: int = 0, _accumulate_step: int = 0, prefix: str = "",
                    hf_enable: bool = False, data_state: Optional[dict] = None,
                    data_coord: Optional[tuple[int, int]] = None) -> None:
    """Write one checkpoint directory.  ``data_state`` (this rank's data-loader position, when the
    loader reports one) is stored beside the rank's RNG state in ``engine/rank_<r>.pt``, with
    ``data_coord`` = (data-parallel rank, data-parallel size) of the stream it belongs to."""
    cur = Path(cur_checkpoint_dir)
    backend = infer_checkpoint_backend(mesh)
    if prefix == "":
        (cur / "engine").mkdir(parents=True, exist_ok=True)
        _barrier()
        per_rank = _rng_state()
        if data_state is not None:
            per_rank["data_state"] = data_state
        if data_coord is not None:
            per_rank["data_coord"] = tuple(int(x) for x in data_coord)
        torch.save(per_rank, cur / "engine" / f"rank_{get_rank()}.pt")

    if backend == "ddp":
        # Unsharded: every rank holds full state; rank 0 writes it.
        msd = model_state_dict(model, full=True) if _is_native(model) else None
        osd = optimizer_state_dict(model, optimizer, full=True) if (optimizer is not None and
                                                                   hasattr(optimizer, "checkpoint_state_dict")) \
            else None
        if is_main_process():
            if msd is None:
                base = _base(model)
                msd = (base.module if hasattr(base, "module") else base).state_dict()
            torch.save(msd, cur / f"{prefix}model.pt")
            if optimizer is not None:
                torch.save(osd if osd is not None else optimizer.state_dict(), cur / f"{prefix}optimizer.pt")
    else:
        msd = model_state_dict(model, full=False)
        dcp.save({"model": msd}, checkpoint_id=str(cur / f"{prefix}model"), process_group=_pg(),
                 storage_writer=dcp.FileSystemWriter(str(cur / f"{prefix}model")))
        del msd
        gc.collect()
        if optimizer is not None:
            osd = optimizer_state_dict(model, optimizer, full=False)
            dcp.save({"optimizer": osd}, checkpoint_id=str(cur / f"{prefix}optimizer"), process_group=_pg(),
                     storage_writer=dcp.FileSystemWriter(str(cur / f"{prefix}optimizer")))
            del osd
            gc.collect()

    if hf_enable:
        save_hf_checkpoint(model, cur / f"{prefix}{HF_MODEL_DIRNAME}")

    if prefix == "" and is_main_process():
        state = {"step": step, "epoch": epoch, "_accumulate_step": _accumulate_step}
        if scheduler is not None:
            state["scheduler"] = scheduler.state_dict()
        if scaler is not None:
            state["scaler"] = scaler.state_dict()
        torch.save(state, cur / "engine.pt")


def save_hf_checkpoint(model: nn.Module, hf_dir: Path) -> None:
    """Full HF-named safetensors from rank 0 (all ranks take part in the gather)."""
    from safetensors.torch import save_file

    full = model_state_dict(model, full=True)
    if not is_main_process():
        return
    Path(hf_dir).mkdir(parents=True, exist_ok=True)
    tensors = {}
    seen: dict[int, str] = {}
    for k, v in full.items():
        if not isinstance(v, torch.Tensor):
            continue
        t = v.detach().to("cpu").contiguous()
        ptr = t.data_ptr()
        if ptr in seen:  # tied weights: safetensors refuses shared storage
            t = t.clone()
        seen[t.data_ptr()] = k
        tensors[k] = t
    save_file(tensors, str(Path(hf_dir) / "model.safetensors"))


# -------------------------------------------------------------------- load
def load_checkpoint(mesh, ckpt_path, model: nn.Module, optimizer=None, scheduler=None, scaler=None,
                    prefix: str = "", restore_engine_state: bool = True, restore_rng_state: bool = True,
                    hf_enable: bool = False, data_coord: Optional[tuple[int, int]] = None) -> Optional[dict[str, int]]:
    cur = Path(ckpt_path)
    backend = infer_checkpoint_backend(mesh)
    base = _base(model)
    has_pt = (cur / f"{prefix}model.pt").exists()
    has_dcp = (cur / f"{prefix}model" / ".metadata").exists()
    hf_path = cur / f"{prefix}{HF_MODEL_DIRNAME}" / "model.safetensors"

    if has_pt or has_dcp:
        if has_pt and (backend == "ddp" or not has_dcp):
            sd = torch.load(cur / f"{prefix}model.pt", map_location="cpu", weights_only=False)
            _load_model_full(base, sd)
            if optimizer is not None and (cur / f"{prefix}optimizer.pt").exists():
                osd = torch.load(cur / f"{prefix}optimizer.pt", map_location="cpu", weights_only=False)
                if hasattr(optimizer, "load_checkpoint_state_dict"):
                    optimizer.load_checkpoint_state_dict(osd, full=True)
                else:
                    optimizer.load_state_dict(osd)
        else:
            msd = model_state_dict(model, full=False)
            holder = {"model": msd}
            dcp.load(holder, checkpoint_id=str(cur / f"{prefix}model"), process_group=_pg())
            if _is_native(base):
                base.load_checkpoint_state_dict(holder["model"], full=False)
            else:
                from torch.distributed.checkpoint.state_dict import set_model_state_dict

                set_model_state_dict(base, holder["model"])
            if optimizer is not None:
                osd = optimizer_state_dict(model, optimizer, full=False)
                holder = {"optimizer": osd}
                dcp.load(holder, checkpoint_id=str(cur / f"{prefix}optimizer"), process_group=_pg())
                if hasattr(optimizer, "load_checkpoint_state_dict"):
                    optimizer.load_checkpoint_state_dict(holder["optimizer"], full=False)
                else:
                    from torch.distributed.checkpoint.state_dict import set_optimizer_state_dict

                    _fill_missing_optimizer_states(base, holder["optimizer"])
                    set_optimizer_state_dict(base, optimizer, holder["optimizer"])
    elif hf_enable and hf_path.exists():
        from safetensors.torch import load_file

        _load_model_full(base, load_file(str(hf_path), device="cpu"))
        return None
    else:
        raise FileNotFoundError(f"Checkpoint not found under {cur} (model.pt, model/.metadata or {hf_path}).")

    if prefix != "" or not restore_engine_state:
        return None
    state = torch.load(cur / "engine.pt", map_location="cpu", weights_only=False)
    if scheduler is not None and "scheduler" in state:
        scheduler.load_state_dict(state["scheduler"])
    if scaler is not None and "scaler" in state:
        scaler.load_state_dict(state["scaler"])
    out = {"step": state["step"], "epoch": state["epoch"], "_accumulate_step": state["_accumulate_step"]}
    own, stream = _per_rank_states(cur, data_coord)
    if own is not None and restore_rng_state:
        _restore_rng(own)
    if stream is not None and "data_state" in stream:
        out["data_state"] = stream["data_state"]
    return out


def _per_rank_states(cur: Path, data_coord: Optional[tuple[int, int]]) -> tuple[Optional[dict], Optional[dict]]:
    """(RNG state to restore, state holding this rank's data position).

    The rank's own file serves both when its data coordinate matches (or either side has none: older
    checkpoints).  After a change of layout -- e.g. a checkpoint of one process resumed by two tensor-parallel
    ranks, which read the same stream -- the data position comes from a file with the same (data-parallel
    rank, size); a rank without a file of its own takes that file's RNG state too.  When no file matches
    (the data-parallel size changed, so the stream is split differently), no position is restored."""
    def read(path: Path) -> Optional[dict]:
        return torch.load(path, map_location="cpu", weights_only=False) if path.exists() else None

    own = read(cur / "engine" / f"rank_{get_rank()}.pt")
    want = tuple(data_coord) if data_coord is not None else None
    if own is not None and (want is None or own.get("data_coord") in (None, want)):
        return own, own
    for path in sorted((cur / "engine").glob("rank_*.pt")):
        other = read(path)
        if other is not None and other.get("data_coord") == want:
            return (own if own is not None else other), other
    if own is not None or want is not None:
        from ..log import simple_info

        simple_info("data-loader position not restored: no checkpointed rank read the same share of the stream "
                    f"(data-parallel rank / size {want})", level="warning")
    return own, None


def _load_model_full(base: nn.Module, sd: dict[str, torch.Tensor]) -> None:
    if _is_native(base):
        base.load_checkpoint_state_dict(sd, full=True)
        return
    target = base.module if hasattr(base, "module") and isinstance(base.module, nn.Module) else base
    try:
        from torch.distributed.fsdp import FSDPModule

        if isinstance(target, FSDPModule):
            from torch.distributed.checkpoint.state_dict import StateDictOptions, set_model_state_dict

            set_model_state_dict(target, sd, options=StateDictOptions(full_state_dict=True, cpu_offload=True,
                                                                       strict=False))
            return
    except ImportError:  # pragma: no cover
        pass
    missing, unexpected = target.load_state_dict(sd, strict=False)
    if missing and is_main_process():
        simple_info(f"checkpoint load: {len(missing)} missing keys (e.g. {missing[:3]})", "warning")
