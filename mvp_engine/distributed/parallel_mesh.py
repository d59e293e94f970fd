"""Named DeviceMesh with semantic roles (reference: mvp_engine/distributed/parallel_mesh.py:38-264).

Mesh dimensions, outermost first: ``replicate``, ``shard``, ``context``,
``tensor``.  One dimension may be ``-1`` and is inferred from the world size.
Roles map to dimension tuples: ``dp``/``fsdp`` = (replicate, shard),
``ddp`` = (replicate,), ``tp``/``sp`` = (tensor,), ``cp`` = (context,).  Unlike
the reference, ``context`` is a real mesh dimension here and drives ring /
Ulysses context parallelism.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Mapping, Optional, Sequence

import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh, init_device_mesh

from ..utils.log import simple_info

DEFAULT_ROLE_DIMS: dict[str, tuple[str, ...]] = {
    "dp": ("replicate", "shard"),
    "ddp": ("replicate",),
    "fsdp": ("replicate", "shard"),
    "tp": ("tensor",),
    "sp": ("tensor",),
    "cp": ("context",),
    "dp_cp": ("replicate", "shard", "context"),
}

MESH_DIM_ORDER = ("replicate", "shard", "context", "tensor")


@dataclass(frozen=True)
class MeshRole:
    name: str
    dim_names: tuple[str, ...]
    mesh: Optional[DeviceMesh]
    group: Optional[dist.ProcessGroup]
    world_size: int
    rank: int
    active: bool


def resolve_mesh_shape(mesh_cfg: Mapping[str, int], world_size: int) -> dict[str, int]:
    """Sizes of every mesh dimension: a ``-1`` (at most one) takes whatever the others leave of ``world_size``.

    The result's product must be ``world_size``; anything else is a configuration error."""
    sizes = {name: int(v) for name, v in mesh_cfg.items()}
    free = [name for name, v in sizes.items() if v == -1]
    if len(free) > 1:
        raise ValueError("Only one device mesh dimension can be inferred.")
    fixed = math.prod(v for v in sizes.values() if v != -1)
    if free:
        quotient, remainder = divmod(world_size, fixed)
        if remainder:
            raise ValueError(f"Cannot infer mesh dimension {free[0]!r}: world_size={world_size} is not divisible "
                             f"by {fixed}.")
        sizes[free[0]] = quotient
    if math.prod(sizes.values()) != world_size:
        raise ValueError(f"Device mesh shape {tuple(sizes.values())} has size {math.prod(sizes.values())}, "
                         f"but world size is {world_size}.")
    return sizes


class ParallelMesh:
    device_mesh: Optional[DeviceMesh]

    @classmethod
    def initialize(cls, device_type: str, mesh_cfg: Mapping[str, int], *,
                   role_dims: Optional[Mapping[str, Sequence[str]]] = None) -> "ParallelMesh":
        world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        ordered = {k: mesh_cfg[k] for k in MESH_DIM_ORDER if k in mesh_cfg}
        ordered.update({k: v for k, v in mesh_cfg.items() if k not in ordered})
        cfg = resolve_mesh_shape(ordered, world)
        simple_info(f"Device Mesh initializing: {' / '.join(cfg)} ({' / '.join(map(str, cfg.values()))})...")
        if dist.is_available() and dist.is_initialized():
            mesh = init_device_mesh(device_type, tuple(cfg.values()), mesh_dim_names=tuple(cfg.keys()))
        else:
            mesh = None
        return cls(mesh, role_dims=role_dims, shape=cfg)

    def __init__(self, device_mesh: Optional[DeviceMesh], *,
                 role_dims: Optional[Mapping[str, Sequence[str]]] = None,
                 shape: Optional[Mapping[str, int]] = None) -> None:
        self.device_mesh = device_mesh
        if device_mesh is not None:
            self.dim_names = tuple(device_mesh.mesh_dim_names or ())
            self._shape = {n: int(device_mesh[n].size()) for n in self.dim_names}
        else:
            self._shape = dict(shape or {})
            self.dim_names = tuple(self._shape)
        self.global_rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
        self.global_world_size = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        self._role_dims = dict(DEFAULT_ROLE_DIMS)
        if role_dims:
            self._role_dims.update({k: tuple(v) for k, v in role_dims.items()})
        self._roles: dict[str, MeshRole] = {}

    # roles -------------------------------------------------------------
    @property
    def dp(self) -> MeshRole:
        return self.role("dp")

    @property
    def ddp(self) -> MeshRole:
        return self.role("ddp")

    @property
    def fsdp(self) -> MeshRole:
        return self.role("fsdp")

    @property
    def tp(self) -> MeshRole:
        return self.role("tp")

    @property
    def sp(self) -> MeshRole:
        return self.role("sp")

    @property
    def cp(self) -> MeshRole:
        return self.role("cp")

    @property
    def dp_cp(self) -> MeshRole:
        """Ranks that share parameters and reduce gradients / token counts: data x context
        parallel (the dp role itself when context parallelism is off)."""
        return self.role("dp_cp") if self.has_dim("context") and self._shape.get("context", 1) > 1 else self.dp

    def role(self, name: str) -> MeshRole:
        cached = self._roles.get(name)
        if cached is not None:
            return cached
        if name in self._role_dims:
            dims = tuple(d for d in self._role_dims[name] if d in self.dim_names)
        elif name in self.dim_names:
            dims = (name,)
        else:
            raise KeyError(f"Unknown mesh role or dimension: {name}")
        size = math.prod(self._shape[d] for d in dims) if dims else 1
        mesh = group = None
        if dims and self.device_mesh is not None:
            mesh = self.device_mesh[dims[0]] if len(dims) == 1 else self.device_mesh[dims]
            if size > 1:
                group = mesh.get_group() if len(dims) == 1 else mesh._flatten("_".join(dims)).get_group()
        rank = dist.get_rank(group) if group is not None else 0
        role = MeshRole(name, dims, mesh, group, size, rank, size > 1)
        self._roles[name] = role
        return role

    def submesh(self, name: str) -> Optional[DeviceMesh]:
        return self.role(name).mesh

    def group(self, name: str) -> Optional[dist.ProcessGroup]:
        return self.role(name).group

    def world_size(self, name: str) -> int:
        return self.role(name).world_size

    def rank(self, name: str) -> int:
        return self.role(name).rank

    def active(self, name: str) -> bool:
        return self.role(name).active

    def has_dim(self, name: str) -> bool:
        return name in self.dim_names

    def dim_size(self, name: str) -> int:
        if not self.has_dim(name):
            raise KeyError(f"Unknown mesh dimension: {name}")
        return self._shape[name]

    def dim_rank(self, name: str) -> int:
        if self.dim_size(name) <= 1 or self.device_mesh is None:
            return 0
        return dist.get_rank(self.device_mesh[name].get_group())

    def summary(self) -> dict[str, Any]:
        roles = {n: self.role(n) for n in DEFAULT_ROLE_DIMS if n != "dp_cp"}
        return {
            "dim_names": self.dim_names,
            "shape": tuple(self._shape[d] for d in self.dim_names),
            "roles": {n: {"dim_names": r.dim_names, "world_size": r.world_size, "rank": r.rank, "active": r.active}
                      for n, r in roles.items()},
        }
