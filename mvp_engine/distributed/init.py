"""Process-group bootstrap (reference: mvp_engine/distributed/init.py:23-66).

Differences from the reference, on purpose:
* CPU runs with world_size > 1 initialise a gloo group (the reference returns
  early on CPU, so it cannot run multi-rank without accelerators);
* every group gets an explicit timeout (``MVP_PG_TIMEOUT_S``, default 600 s)
  so a rank that dies or never joins ends the others' collectives with an
  error instead of a hang.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist

from .utils import configure_distributed_socket_ifnames, get_local_rank


def _backend_for(device_type: str) -> str:
    return "nccl" if device_type == "cuda" else "gloo"


def pg_timeout() -> timedelta:
    return timedelta(seconds=float(os.environ.get("MVP_PG_TIMEOUT_S", "600")))


def initialize_process_group(backend: str | None = None) -> None:
    """Initialise torch.distributed from RANK/WORLD_SIZE/MASTER_* (env://) if not done yet."""
    if dist.is_initialized():
        return
    world_size = int(os.getenv("WORLD_SIZE", "1"))
    rank = int(os.getenv("RANK", "0"))
    if world_size <= 0:
        raise ValueError("WORLD_SIZE must be greater than 0 for distributed training.")
    if torch.cuda.is_available():
        device_type = "cuda"
        torch.cuda.set_device(get_local_rank() % max(1, torch.cuda.device_count()))
    else:
        device_type = "cpu"
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    if world_size > 1:
        configure_distributed_socket_ifnames(device_type)
    kwargs = {}
    if device_type == "cuda":
        kwargs["device_id"] = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group(
        backend=backend or _backend_for(device_type),
        init_method="env://",
        world_size=world_size,
        rank=rank,
        timeout=pg_timeout(),
        **kwargs,
    )


def destroy_process_group() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
