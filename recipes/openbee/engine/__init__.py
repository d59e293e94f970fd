from .openbee_engine import OpenBeeEngine

__all__ = ["OpenBeeEngine"]
