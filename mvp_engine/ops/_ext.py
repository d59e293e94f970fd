"""Loader for the in-tree sm_100a extension ``mvp_engine._C``.

The extension is built in place by ``python setup.py build_ext --inplace``
(``__graft_entry__.build`` does the same).  On a machine with a CUDA device the
native path is mandatory: a missing or stale extension raises instead of
silently falling back to eager PyTorch.
"""

from __future__ import annotations

import importlib
import os

import torch

_EXT = None
_ERR: Exception | None = None


def native_required() -> bool:
    """Native kernels are required whenever CUDA is usable (override: MVP_ALLOW_EAGER=1)."""
    return torch.cuda.is_available() and os.environ.get("MVP_ALLOW_EAGER", "0") != "1"


def ext():
    """Return the loaded extension module, importing it on first use."""
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    try:
        _EXT = importlib.import_module("mvp_engine._C")
    except Exception as exc:  # pragma: no cover - depends on the build
        _ERR = exc
        raise RuntimeError(
            "mvp_engine._C is not built; run `python setup.py build_ext --inplace` at the repo root"
        ) from exc
    return _EXT


def available() -> bool:
    """True when the extension imports and a CUDA device is present."""
    if not torch.cuda.is_available():
        return False
    try:
        ext()
        return True
    except RuntimeError:
        return False


_STATUS: dict[int, torch.Tensor] = {}


def status_buffer(device: torch.device | int | None = None) -> torch.Tensor:
    """Per-device int32 status word that bounded device-side waits write on timeout."""
    if device is None:
        device = torch.cuda.current_device()
    index = device.index if isinstance(device, torch.device) else int(device)
    buf = _STATUS.get(index)
    if buf is None:
        buf = torch.zeros(4, dtype=torch.int32, device=f"cuda:{index}")
        _STATUS[index] = buf
    return buf


def check_status(device: torch.device | int | None = None, reset: bool = True) -> int:
    """Read (and optionally clear) the device status word; raise if a kernel timed out."""
    buf = status_buffer(device)
    code = int(buf[0].item())
    if code != 0:
        if reset:
            buf.zero_()
        raise RuntimeError(f"mvp_engine kernel reported status {code} (bounded wait expired)")
    return code
