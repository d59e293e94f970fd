"""Log backends: terminal, file, wandb."""

from .backend import Backend
from .file import FileBackend
from .terminal import TerminalBackend
from .wandb import WandbBackend

__all__ = ["Backend", "FileBackend", "TerminalBackend", "WandbBackend"]
