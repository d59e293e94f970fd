"""Step tracing: NVTX ranges per engine phase and per block, and an opt-in ``torch.profiler`` window.

The reference times steps with host wall-clock scopes only (``mvp_engine/utils/log/timer.py:60-87``) and
carries one ``record_function`` label (``mvp_engine/patches/torch_fsdp2.py:83``).  This engine adds, all
off by default and configured under ``trace:``:

* ``nvtx``: one NVTX range per micro-batch phase (``data``, ``forward``, ``backward``, ``optimizer``),
  nested under a ``step_<n>`` range per optimizer step.  ``ncu --nvtx --nvtx-include`` and Nsight
  Systems select kernels by these names.  ``MVP_NVTX=1`` in the environment turns it on without a
  config change.
* ``nvtx_blocks``: one range per forward call of each transformer block (modules whose class name is in
  ``block_classes``, default: names ending in ``DecoderLayer`` or ``Block``), attached with forward hooks
  so the model code is untouched.  Backward work of a block runs on autograd's thread and shows up
  inside the ``backward`` range.
* ``profiler``: a ``torch.profiler`` schedule (``wait`` / ``warmup`` / ``active`` optimizer steps,
  ``repeat`` windows) writing one Chrome trace per window and rank to
  ``<run output dir>/profile/rank<r>_step<n>.json``.  The phase names above are also emitted as
  ``record_function`` labels while a window records.

When everything is off, :meth:`StepTracer.range` hands back one shared ``nullcontext``: the hot loop pays
an attribute lookup and a call per phase.
"""

from __future__ import annotations

import contextlib
import os
import re
from pathlib import Path
from typing import Any, Iterator, Optional

import torch
from pydantic import BaseModel, ConfigDict, Field

_NULL = contextlib.nullcontext()


class ProfilerConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    enabled: bool = False
    wait: int = Field(1, ge=0)  # optimizer steps skipped before each window
    warmup: int = Field(1, ge=0)  # steps traced but discarded (profiler start-up cost)
    active: int = Field(2, ge=1)  # steps recorded per window
    repeat: int = Field(1, ge=0)  # windows; 0 = until training ends
    record_shapes: bool = False
    with_stack: bool = False
    profile_memory: bool = False


class TraceConfig(BaseModel):
    model_config = ConfigDict(frozen=False)

    nvtx: bool = False
    nvtx_blocks: bool = False
    block_classes: list[str] = []
    profiler: ProfilerConfig = Field(default_factory=ProfilerConfig)


def _env_flag(name: str) -> bool:
    return os.environ.get(name, "").strip().lower() in ("1", "true", "yes", "on")


class StepTracer:
    """Per-engine tracing state; see the module docstring for what each switch emits."""

    def __init__(self, config: Optional[TraceConfig] = None, out_dir: Optional[Path] = None, rank: int = 0):
        self.config = config or TraceConfig()
        self.nvtx = bool(self.config.nvtx or _env_flag("MVP_NVTX"))
        self.rank = int(rank)
        self.out_dir = Path(out_dir) if out_dir is not None else None
        self.traces: list[Path] = []
        self._hooks: list[Any] = []
        self._profiler = None
        self._step_open = False
        if self.config.profiler.enabled:
            self._profiler = self._start_profiler()

    @classmethod
    def disabled(cls) -> "StepTracer":
        """A tracer that emits nothing, whatever the environment says."""
        t = cls(TraceConfig())
        t.nvtx = False
        return t

    @property
    def enabled(self) -> bool:
        return self.nvtx or self._profiler is not None

    # ---------------------------------------------------------------- ranges
    @contextlib.contextmanager
    def _range(self, name: str) -> Iterator[None]:
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        label = torch.profiler.record_function(name) if self._profiler is not None else _NULL
        try:
            with label:
                yield
        finally:
            if self.nvtx:
                torch.cuda.nvtx.range_pop()

    def range(self, name: str):
        """Context manager around one phase; a shared no-op when tracing is off."""
        return self._range(name) if self.enabled else _NULL

    def begin_step(self, step: int) -> None:
        """Open the ``step_<n>`` range (once per optimizer step, before its first micro-batch)."""
        if self.nvtx and not self._step_open:
            torch.cuda.nvtx.range_push(f"step_{step}")
            self._step_open = True

    def end_step(self, step: int) -> None:
        """Close the step range and advance the profiler schedule (after the optimizer step)."""
        if self._step_open:
            torch.cuda.nvtx.range_pop()
            self._step_open = False
        if self._profiler is not None:
            self._profiler.step()

    # ---------------------------------------------------------------- blocks
    def _is_block(self, module: torch.nn.Module) -> bool:
        name = type(module).__name__
        if self.config.block_classes:
            return name in self.config.block_classes
        return name.endswith("DecoderLayer") or name.endswith("Block")

    def attach_blocks(self, model: torch.nn.Module) -> int:
        """NVTX range around the forward of every block of ``model``; returns how many were hooked."""
        if not (self.nvtx and self.config.nvtx_blocks):
            return 0
        for fqn, module in model.named_modules():
            if not self._is_block(module):
                continue
            label = re.sub(r"^(_orig_mod\.|module\.)+", "", fqn) or type(module).__name__

            def push(_m, _args, _label=label):
                torch.cuda.nvtx.range_push(_label)

            def pop(_m, _args, _out):
                torch.cuda.nvtx.range_pop()

            self._hooks.append(module.register_forward_pre_hook(push))
            self._hooks.append(module.register_forward_hook(pop))
        return len(self._hooks) // 2

    # -------------------------------------------------------------- profiler
    def _start_profiler(self):
        from torch.profiler import ProfilerActivity, profile, schedule

        cfg = self.config.profiler
        activities = [ProfilerActivity.CPU]
        if torch.cuda.is_available():
            activities.append(ProfilerActivity.CUDA)
        prof = profile(activities=activities,
                       schedule=schedule(wait=cfg.wait, warmup=cfg.warmup, active=cfg.active, repeat=cfg.repeat),
                       on_trace_ready=self._export, record_shapes=cfg.record_shapes, with_stack=cfg.with_stack,
                       profile_memory=cfg.profile_memory)
        prof.start()
        return prof

    def _export(self, prof) -> None:
        if self.out_dir is None:
            return
        self.out_dir.mkdir(parents=True, exist_ok=True)
        path = self.out_dir / f"rank{self.rank}_step{prof.step_num}.json"
        prof.export_chrome_trace(str(path))
        self.traces.append(path)

    def close(self) -> None:
        if self._step_open:
            torch.cuda.nvtx.range_pop()
            self._step_open = False
        for h in self._hooks:
            h.remove()
        self._hooks.clear()
        if self._profiler is not None:
            self._profiler.stop()
            self._profiler = None
