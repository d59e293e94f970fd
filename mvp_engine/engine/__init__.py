"""Engine base class, step context and the engine registry."""

from ..utils.registry import Registry

ENGINE_REGISTRY = Registry("engine")

from .engine import Engine, TrainStepContext  # noqa: E402

ENGINE_REGISTRY.register()(Engine)

__all__ = ["ENGINE_REGISTRY", "Engine", "TrainStepContext"]
