"""Rank helpers, NIC selection for gloo/NCCL sockets, and rank-0 object broadcast
(reference: mvp_engine/distributed/utils.py:12-167)."""

from __future__ import annotations

import os
import pickle
import socket
from typing import Any, Optional

import torch
import torch.distributed as dist


def get_rank() -> int:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank()
    return int(os.environ.get("RANK", "0"))


def get_local_rank() -> int:
    return int(os.getenv("LOCAL_RANK", str(get_rank())))


def get_world_size() -> int:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size()
    return 1


def is_main_process() -> bool:
    return get_rank() == 0


def _iface_up(name: str) -> bool:
    try:
        with open(f"/sys/class/net/{name}/operstate") as f:
            return f.read().strip() in ("up", "unknown")
    except OSError:
        return False


def guess_socket_interface() -> Optional[str]:
    """Pick the interface that routes to MASTER_ADDR (UDP connect trick), else a non-loopback one that is up."""
    master = os.environ.get("MASTER_ADDR")
    if master:
        try:
            s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
            try:
                s.connect((master, int(os.environ.get("MASTER_PORT", "29500"))))
                local_ip = s.getsockname()[0]
            finally:
                s.close()
            for _, name in socket.if_nameindex():
                if _iface_ip(name) == local_ip:
                    return name
        except OSError:
            pass
    candidates = []
    for _, name in socket.if_nameindex():
        if name == "lo" or not _iface_up(name):
            continue
        score = 0 if name.startswith(("docker", "veth", "br-", "virbr")) else 1
        candidates.append((score, name))
    candidates.sort(reverse=True)
    return candidates[0][1] if candidates else None


def _iface_ip(name: str) -> Optional[str]:
    try:
        import fcntl
        import struct

        s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        try:
            packed = fcntl.ioctl(s.fileno(), 0x8915, struct.pack("256s", name[:15].encode()))
            return socket.inet_ntoa(packed[20:24])
        finally:
            s.close()
    except OSError:
        return None


def configure_distributed_socket_ifnames(device_type: str) -> dict[str, str]:
    """Fill GLOO_SOCKET_IFNAME (and NCCL_SOCKET_IFNAME on CUDA) when unset. Loopback rendezvous
    (MASTER_ADDR=127.0.0.1, single node) keeps the default so local runs stay on ``lo``."""
    names = ["GLOO_SOCKET_IFNAME"] + (["NCCL_SOCKET_IFNAME"] if device_type == "cuda" else [])
    configured: dict[str, str] = {}
    if os.environ.get("MASTER_ADDR", "127.0.0.1") in ("127.0.0.1", "localhost"):
        return {n: os.environ[n] for n in names if os.environ.get(n)}
    guess = None
    for n in names:
        if os.environ.get(n):
            configured[n] = os.environ[n]
            continue
        guess = guess or guess_socket_interface()
        if guess:
            os.environ[n] = guess
            configured[n] = guess
    return configured


_GLOO_WORLD: Optional[dist.ProcessGroup] = None


def gloo_world_group() -> Optional[dist.ProcessGroup]:
    """A lazily created gloo group over all ranks (host-side object exchange)."""
    global _GLOO_WORLD
    if not dist.is_initialized():
        return None
    if dist.get_backend() == "gloo":
        return dist.group.WORLD
    if _GLOO_WORLD is None:
        _GLOO_WORLD = dist.new_group(backend="gloo")
    return _GLOO_WORLD


def broadcast_from_main(obj: Any, group: Optional[dist.ProcessGroup] = None) -> Any:
    """Pickle ``obj`` on rank 0 and return it on every rank (over gloo)."""
    if not (dist.is_available() and dist.is_initialized()) or get_world_size() == 1:
        return obj
    group = group or gloo_world_group()
    payload = [obj if get_rank() == 0 else None]
    dist.broadcast_object_list(payload, src=0, group=group)
    return payload[0]


def all_gather_objects(obj: Any, group: Optional[dist.ProcessGroup] = None) -> list:
    if not (dist.is_available() and dist.is_initialized()) or get_world_size() == 1:
        return [obj]
    group = group or gloo_world_group()
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out
