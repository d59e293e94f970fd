"""Small helpers (reference: mvp_engine/utils/misc.py:1-69)."""

from __future__ import annotations

import subprocess

import torch
import torch.nn as nn


def freeze(module: nn.Module) -> None:
    """Put ``module`` in eval mode and stop gradients to all of its parameters."""
    module.eval()
    for p in module.parameters():
        p.requires_grad = False


def find_optimizable_params(module: nn.Module):
    """Yield the parameters of ``module`` that require grad."""
    return (p for p in module.parameters() if p.requires_grad)


def get_device(index: int = 0) -> torch.device:
    """``cuda:<index>`` when CUDA is usable, else ``cpu``."""
    if torch.cuda.is_available():
        return torch.device(f"cuda:{index}")
    return torch.device("cpu")


def _git(*args: str) -> str:
    try:
        return subprocess.check_output(["git", *args], stderr=subprocess.DEVNULL).decode().strip()
    except (subprocess.CalledProcessError, FileNotFoundError, OSError):
        return "None"


def get_git_info() -> dict[str, str]:
    """Current branch and commit hash (``"None"`` outside a git checkout)."""
    return {"branch": _git("rev-parse", "--abbrev-ref", "HEAD"), "commit_hash": _git("rev-parse", "HEAD")}


def calculate_model_size(model: nn.Module) -> tuple[int, int]:
    """Return ``(total, trainable)`` parameter counts (logical, unsharded when known)."""
    counter = getattr(model, "logical_parameter_counts", None)
    if callable(counter):
        return counter()
    total = sum(p.numel() for p in model.parameters())
    trainable = sum(p.numel() for p in model.parameters() if p.requires_grad)
    return total, trainable
