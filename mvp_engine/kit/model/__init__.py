from .liger import LigerKernelKit, LigerKernelReport, LigerPatch

__all__ = ["LigerKernelKit", "LigerKernelReport", "LigerPatch"]
