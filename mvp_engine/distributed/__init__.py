"""Distributed bootstrap, meshes and model wrapping."""

__all__ = ["MeshRole", "ParallelMesh"]


def __getattr__(name: str):
    if name in __all__:
        from . import parallel_mesh

        return getattr(parallel_mesh, name)
    raise AttributeError(name)
