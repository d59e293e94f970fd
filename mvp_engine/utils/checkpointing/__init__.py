"""Checkpoint I/O."""

from .parallel_sl_util import load_checkpoint, save_checkpoint, save_hf_checkpoint

__all__ = ["save_checkpoint", "load_checkpoint", "save_hf_checkpoint"]
