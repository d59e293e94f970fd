"""Model-FLOPs utilisation for training logs.

Public API and log key of the reference's ``MFUKit`` (``mvp_engine/kit/perf/mfu.py:14-230``
there); the definition is the same so numbers compare::

    perf/mfu = sum over ranks of model FLOPs in the step
               / (max over ranks of the step time x peak FLOP/s x world size)

The reference's peak table has no B200 row, so its ``perf/mfu`` is empty on
B200; this table adds B200 at its dense figures.  Peaks are kept as a small
text table (device, precision, TFLOP/s) plus substring rules that map the
names CUDA / nvidia-smi report onto the table's device names.  A caller can
also pass a measured peak (``configured_peak_tflops``), and the environment
variable ``MVP_PEAK_TFLOPS`` overrides the table for every call.
"""

from __future__ import annotations

import os
import subprocess
from typing import Any, Optional

import torch
import torch.distributed as dist

from ...distributed.utils import get_world_size

_PEAK_TABLE = """
NVIDIA B200        bf16 2250
NVIDIA B200        fp16 2250
NVIDIA B200        fp8  4500
NVIDIA B200        tf32 1125
NVIDIA B200        fp32 75
NVIDIA H200        bf16 989
NVIDIA H200        fp16 989
NVIDIA H100 SXM    bf16 989
NVIDIA H100 SXM    fp16 989
NVIDIA H100 PCIe   bf16 756
NVIDIA H100 PCIe   fp16 756
NVIDIA A100 80GB   bf16 312
NVIDIA A100 80GB   fp16 312
NVIDIA A100 40GB   bf16 312
NVIDIA A100 40GB   fp16 312
NVIDIA L40S        bf16 733
NVIDIA L40S        fp16 733
NVIDIA RTX 4090    bf16 330
NVIDIA RTX 4090    fp16 330
"""

# (substring of the upper-cased reported name, table device name); first match wins
_NAME_RULES = (
    ("B200", "NVIDIA B200"), ("H200", "NVIDIA H200"), ("H100 PCIE", "NVIDIA H100 PCIe"),
    ("H100 SXM", "NVIDIA H100 SXM"), ("H100 80GB HBM3", "NVIDIA H100 SXM"), ("A100-SXM4-80GB", "NVIDIA A100 80GB"),
    ("A100 80GB", "NVIDIA A100 80GB"), ("A100 40GB", "NVIDIA A100 40GB"), ("L40S", "NVIDIA L40S"),
    ("RTX 4090", "NVIDIA RTX 4090"),
)


def _parse_peaks(text: str) -> dict[tuple[str, str], float]:
    table = {}
    for line in text.strip().splitlines():
        *device, precision, tflops = line.split()
        table[(" ".join(device), precision)] = float(tflops)
    return table


def _positive(**named: float) -> None:
    for key, val in named.items():
        if not val > 0:
            raise ValueError(f"{key} must be > 0")


class MFUKit:
    PEAK_TFLOPS_BY_DEVICE_AND_PRECISION: dict[tuple[str, str], float] = _parse_peaks(_PEAK_TABLE)

    def __init__(self) -> None:
        self._accumulated_model_flops = 0.0

    @property
    def accumulated_model_flops(self) -> float:
        """Model FLOPs recorded by :meth:`accumulate_microbatch` since the last reset (this rank)."""
        return self._accumulated_model_flops

    def reset(self) -> None:
        self._accumulated_model_flops = 0.0

    @staticmethod
    def _model_flops(model: Any, batch_size: Optional[int], seq_len: Optional[int], **kw: Any) -> float:
        if model is None or batch_size is None or seq_len is None:
            raise ValueError("Either model_flops or model/batch_size/seq_len must be provided.")
        return float(model.calculate_model_flops(batch_size=int(batch_size), seq_len=int(seq_len), **kw))

    def accumulate_microbatch(self, *, model_flops: Optional[float] = None, model: Any = None,
                              batch_size: Optional[int] = None, seq_len: Optional[int] = None, **kw: Any) -> float:
        """Add one micro-batch's model FLOPs (given, or from ``model.calculate_model_flops``)."""
        flops = float(model_flops) if model_flops is not None else self._model_flops(model, batch_size, seq_len, **kw)
        if flops < 0:
            raise ValueError("model_flops must be non-negative.")
        self._accumulated_model_flops += flops
        return flops

    def calculate_mfu(self, *, model_flops_per_step: float, step_time_seconds: float, device_peak_tflops: float,
                      world_size: int) -> float:
        _positive(step_time_seconds=step_time_seconds, device_peak_tflops=device_peak_tflops, world_size=world_size)
        achieved = model_flops_per_step / step_time_seconds
        return float(achieved / (device_peak_tflops * 1e12 * world_size))

    def reduce_to_global_flops_and_step_time(self, *, model_flops_per_step: float,
                                             step_time_seconds: float) -> tuple[float, float]:
        """(sum of FLOPs over ranks, max step time over ranks); identity without a process group."""
        if not (dist.is_available() and dist.is_initialized()):
            return float(model_flops_per_step), float(step_time_seconds)
        on = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
        flops = torch.tensor([float(model_flops_per_step)], dtype=torch.float64, device=on)
        secs = torch.tensor([float(step_time_seconds)], dtype=torch.float64, device=on)
        dist.all_reduce(flops, op=dist.ReduceOp.SUM)
        dist.all_reduce(secs, op=dist.ReduceOp.MAX)
        return float(flops.item()), float(secs.item())

    def normalize_device_name(self, device_name: str) -> Optional[str]:
        name = (device_name or "").strip()
        if not name:
            return None
        upper = name.upper()
        return next((canon for needle, canon in _NAME_RULES if needle in upper), name)

    def detect_cuda_device_name(self) -> Optional[str]:
        if torch.cuda.is_available():
            return self.normalize_device_name(torch.cuda.get_device_name(torch.cuda.current_device()))
        try:
            listing = subprocess.run(["nvidia-smi", "--query-gpu=name", "--format=csv,noheader"], check=True,
                                     capture_output=True, text=True).stdout
        except (FileNotFoundError, subprocess.CalledProcessError):
            return None
        names = [ln.strip() for ln in listing.splitlines() if ln.strip()]
        return self.normalize_device_name(names[0]) if names else None

    def resolve_peak_tflops(self, *, device_type: str, precision: str, configured_device_name: Optional[str] = None,
                            configured_peak_tflops: Optional[float] = None) -> tuple[Optional[str], Optional[float]]:
        """(device name, peak TFLOP/s) for the MFU denominator; either may be None when unknown."""
        name = self.normalize_device_name(configured_device_name) if configured_device_name else None
        override = configured_peak_tflops
        if override is None and os.environ.get("MVP_PEAK_TFLOPS"):
            override = float(os.environ["MVP_PEAK_TFLOPS"])
        if override is not None:
            return name, float(override)
        if name is None and device_type == "cuda":
            name = self.detect_cuda_device_name()
        peak = self.PEAK_TFLOPS_BY_DEVICE_AND_PRECISION.get((name, precision)) if name else None
        return name, peak

    def build_log(self, *, model_flops_per_step: Optional[float] = None, model: Any = None, device_type: str,
                  precision: str, batch_size: Optional[int] = None, seq_len: Optional[int] = None,
                  step_time_seconds: float, gradient_accumulation_steps: int = 1,
                  configured_device_name: Optional[str] = None, configured_peak_tflops: Optional[float] = None,
                  **kw: Any) -> dict[str, float]:
        """``{"perf/mfu": value}`` for one optimizer step, or ``{}`` when no peak is known (a configured
        peak counts even when the device name is unknown, unlike the reference).

        The step's FLOPs come from (in this order) ``model_flops_per_step``, the model's formula times
        the accumulation steps, or the micro-batches accumulated since the last call (which this call
        then clears).  Every rank must call it: the FLOPs and the step time are reduced across ranks."""
        from_window = model_flops_per_step is None and model is None
        if step_time_seconds <= 0:
            if from_window:
                self.reset()
            return {}
        if model_flops_per_step is not None:
            local = float(model_flops_per_step)
        elif model is not None and batch_size is not None and seq_len is not None:
            local = self._model_flops(model, batch_size, seq_len, **kw) * int(gradient_accumulation_steps)
        elif self._accumulated_model_flops > 0:
            local = self._accumulated_model_flops
        else:
            raise ValueError("No model FLOPs are available for MFU logging.")
        if from_window:
            self.reset()
        name, peak = self.resolve_peak_tflops(device_type=device_type, precision=precision,
                                              configured_device_name=configured_device_name,
                                              configured_peak_tflops=configured_peak_tflops)
        if peak is None:  # unknown device or precision: nothing to divide by
            return {}
        total, slowest = self.reduce_to_global_flops_and_step_time(model_flops_per_step=local,
                                                                   step_time_seconds=float(step_time_seconds))
        return {"perf/mfu": self.calculate_mfu(model_flops_per_step=total, step_time_seconds=slowest,
                                               device_peak_tflops=peak, world_size=int(get_world_size()))}
