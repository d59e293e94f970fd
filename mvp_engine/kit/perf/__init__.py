from .mfu import MFUKit

__all__ = ["MFUKit"]
