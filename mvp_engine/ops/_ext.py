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

# Kernels launched per extension call (for launch accounting in benchmarks).
KERNELS_PER_CALL = {
    "gemm": 1, "rmsnorm_fwd": 1, "rmsnorm_bwd": 2, "qk_norm_rope_fwd": 1, "qk_norm_rope_bwd": 1, "swiglu_fwd": 1,
    "swiglu_bwd": 1, "ce_fwd": 1, "ce_bwd_": 1, "adamw_step_": 1, "sumsq": 1, "embedding_fwd": 1,
    "embedding_bwd_": 1, "flash_attn_fwd": 1, "flash_attn_bwd": 3, "peer_reduce_scatter": 1, "peer_barrier": 1,
    "peer_push_rows": 2, "peer_wait_all": 1, "peer_slot_reduce": 1, "gemm_pair_tp": 1,
    "peer_publish": 1, "peer_slot_sum_f32": 1, "gemm_ulysses": 1,
    "layernorm_fwd": 1, "layernorm_bwd": 3, "bias_gelu_fwd": 1, "bias_gelu_bwd": 2, "vision_rope_fwd": 1,
    "vision_rope_bwd": 1, "bias_residual_fwd": 1, "bias_grad": 2,
    "peer_gather_shards": 1, "publish_epoch": 1, "gemm_pair_gather": 1,
}
launch_count = 0
counting = False


class _Counting:
    """Forwards to the extension module and counts native kernel launches while enabled."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        k = KERNELS_PER_CALL.get(name)
        if k is None or not callable(fn):
            return fn

        def wrapped(*a, **kw):
            global launch_count
            if counting:
                launch_count += k
            return fn(*a, **kw)

        return wrapped


def start_counting() -> None:
    global counting, launch_count
    counting, launch_count = True, 0


def stop_counting() -> int:
    global counting
    counting = False
    return launch_count


def native_required() -> bool:
    """Native kernels are required whenever CUDA is usable (override: MVP_ALLOW_EAGER=1)."""
    return torch.cuda.is_available() and os.environ.get("MVP_ALLOW_EAGER", "0") != "1"


def ext():
    """Return the loaded extension module, importing it on first use."""
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    try:
        _EXT = _Counting(importlib.import_module("mvp_engine._C"))
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
        what = {6: "bad argument", 7: "bounds check failed (debug build)"}.get(code, "bounded wait expired")
        raise RuntimeError(f"mvp_engine kernel reported status {code} ({what})")
    return code
