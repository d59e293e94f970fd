"""Model-FLOPs utilisation (reference: mvp_engine/kit/perf/mfu.py:14-230).

``perf/mfu = sum_ranks(model FLOPs per step) / (max_ranks(step time) * peak * world)``.
The reference's peak table has no B200 row (so its MFU log is empty there);
this one adds B200 at the dense figures (bf16/fp16 2250, fp8 4500, tf32 1125
TFLOP/s).  A measured peak (``MEASURED_PEAKS.json``-style dict with
``bf16_tflops``) can be supplied instead with ``configured_peak_tflops``.
"""

from __future__ import annotations

import subprocess
from typing import Any, Optional

import torch
import torch.distributed as dist

from ...distributed.utils import get_world_size


class MFUKit:
    PEAK_TFLOPS_BY_DEVICE_AND_PRECISION = {
        ("NVIDIA B200", "bf16"): 2250.0,
        ("NVIDIA B200", "fp16"): 2250.0,
        ("NVIDIA B200", "fp8"): 4500.0,
        ("NVIDIA B200", "tf32"): 1125.0,
        ("NVIDIA B200", "fp32"): 75.0,
        ("NVIDIA H100 SXM", "bf16"): 989.0,
        ("NVIDIA H100 SXM", "fp16"): 989.0,
        ("NVIDIA H100 PCIe", "bf16"): 756.0,
        ("NVIDIA H100 PCIe", "fp16"): 756.0,
        ("NVIDIA H200", "bf16"): 989.0,
        ("NVIDIA H200", "fp16"): 989.0,
        ("NVIDIA A100 80GB", "bf16"): 312.0,
        ("NVIDIA A100 80GB", "fp16"): 312.0,
        ("NVIDIA A100 40GB", "bf16"): 312.0,
        ("NVIDIA A100 40GB", "fp16"): 312.0,
        ("NVIDIA L40S", "bf16"): 733.0,
        ("NVIDIA L40S", "fp16"): 733.0,
        ("NVIDIA RTX 4090", "bf16"): 330.0,
        ("NVIDIA RTX 4090", "fp16"): 330.0,
    }
    _MARKERS = (("B200", "NVIDIA B200"), ("H200", "NVIDIA H200"), ("H100 SXM", "NVIDIA H100 SXM"),
                ("H100 PCIE", "NVIDIA H100 PCIe"), ("H100 80GB HBM3", "NVIDIA H100 SXM"),
                ("A100 80GB", "NVIDIA A100 80GB"), ("A100-SXM4-80GB", "NVIDIA A100 80GB"),
                ("A100 40GB", "NVIDIA A100 40GB"), ("L40S", "NVIDIA L40S"), ("RTX 4090", "NVIDIA RTX 4090"))

    def __init__(self) -> None:
        self.reset()

    def reset(self) -> None:
        self._accumulated_model_flops = 0.0

    def accumulate_microbatch(self, *, model_flops: Optional[float] = None, model: Any = None,
                              batch_size: Optional[int] = None, seq_len: Optional[int] = None, **kw: Any) -> float:
        f = model_flops
        if f is None:
            if model is None or batch_size is None or seq_len is None:
                raise ValueError("Either model_flops or model/batch_size/seq_len must be provided.")
            f = model.calculate_model_flops(batch_size=int(batch_size), seq_len=int(seq_len), **kw)
        if f < 0:
            raise ValueError("model_flops must be non-negative.")
        self._accumulated_model_flops += float(f)
        return float(f)

    def calculate_mfu(self, *, model_flops_per_step: float, step_time_seconds: float, device_peak_tflops: float,
                      world_size: int) -> float:
        if step_time_seconds <= 0:
            raise ValueError("step_time_seconds must be > 0")
        if device_peak_tflops <= 0:
            raise ValueError("device_peak_tflops must be > 0")
        if world_size <= 0:
            raise ValueError("world_size must be > 0")
        return float(model_flops_per_step / step_time_seconds / (device_peak_tflops * 1e12 * world_size))

    def reduce_to_global_flops_and_step_time(self, *, model_flops_per_step: float,
                                             step_time_seconds: float) -> tuple[float, float]:
        if not (dist.is_available() and dist.is_initialized()):
            return float(model_flops_per_step), float(step_time_seconds)
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
        f = torch.tensor([float(model_flops_per_step)], dtype=torch.float64, device=dev)
        t = torch.tensor([float(step_time_seconds)], dtype=torch.float64, device=dev)
        dist.all_reduce(f, op=dist.ReduceOp.SUM)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(f.item()), float(t.item())

    def normalize_device_name(self, device_name: str) -> Optional[str]:
        name = device_name.strip()
        if not name:
            return None
        up = name.upper()
        for marker, canon in self._MARKERS:
            if marker in up:
                return canon
        return name

    def detect_cuda_device_name(self) -> Optional[str]:
        if torch.cuda.is_available():
            return self.normalize_device_name(torch.cuda.get_device_name(torch.cuda.current_device()))
        try:
            out = subprocess.run(["nvidia-smi", "--query-gpu=name", "--format=csv,noheader"], check=True,
                                 capture_output=True, text=True).stdout
        except (FileNotFoundError, subprocess.CalledProcessError):
            return None
        first = next((ln.strip() for ln in out.splitlines() if ln.strip()), None)
        return self.normalize_device_name(first) if first else None

    def resolve_peak_tflops(self, *, device_type: str, precision: str, configured_device_name: Optional[str] = None,
                            configured_peak_tflops: Optional[float] = None) -> tuple[Optional[str], Optional[float]]:
        name = self.normalize_device_name(configured_device_name) if configured_device_name else None
        if configured_peak_tflops is not None:
            return name, float(configured_peak_tflops)
        if name is None and device_type == "cuda":
            name = self.detect_cuda_device_name()
        if name is None:
            return None, None
        peak = self.PEAK_TFLOPS_BY_DEVICE_AND_PRECISION.get((name, precision))
        return name, (float(peak) if peak is not None else None)

    def build_log(self, *, model_flops_per_step: Optional[float] = None, model: Any = None, device_type: str,
                  precision: str, batch_size: Optional[int] = None, seq_len: Optional[int] = None,
                  step_time_seconds: float, gradient_accumulation_steps: int = 1,
                  configured_device_name: Optional[str] = None, configured_peak_tflops: Optional[float] = None,
                  **kw: Any) -> dict[str, float]:
        if step_time_seconds <= 0:
            if model_flops_per_step is None and model is None:
                self.reset()
            return {}
        local = model_flops_per_step
        if local is None:
            if model is not None and batch_size is not None and seq_len is not None:
                local = model.calculate_model_flops(batch_size=int(batch_size), seq_len=int(seq_len), **kw) * int(
                    gradient_accumulation_steps)
            elif self._accumulated_model_flops > 0:
                local = self._accumulated_model_flops
            else:
                raise ValueError("No model FLOPs are available for MFU logging.")
        if model_flops_per_step is None and model is None:
            self.reset()
        name, peak = self.resolve_peak_tflops(device_type=device_type, precision=precision,
                                              configured_device_name=configured_device_name,
                                              configured_peak_tflops=configured_peak_tflops)
        if name is None or peak is None:
            return {}
        gf, gt = self.reduce_to_global_flops_and_step_time(model_flops_per_step=float(local),
                                                           step_time_seconds=float(step_time_seconds))
        return {"perf/mfu": self.calculate_mfu(model_flops_per_step=gf, step_time_seconds=gt,
                                               device_peak_tflops=peak, world_size=int(get_world_size()))}
