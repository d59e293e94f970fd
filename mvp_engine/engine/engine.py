"""Template-method training engine (reference: mvp_engine/engine/engine.py:50-592).

Workflow::

    __init__  : prepare_config -> prepare_parallel -> prepare_runtime_info
                -> set_seed -> prepare_logger
    train()   : before_train -> do_train -> after_train
    do_train  : per micro-batch  train_pre_step -> train_exec_step
                (forward_step -> backward_step -> optimizer_step)
                and after each optimizer step train_post_step + save

Subclasses implement ``prepare_model / prepare_optimizer / prepare_scheduler /
prepare_dataloader`` exactly as in the reference.  Additions of this engine:

* the process group also comes up on CPU (gloo) and always has a timeout;
* every optimizer step is timed on the device with CUDA events
  (``self.step_time_ms``, max over ranks), next to the reference's host
  ``Timer``;
* after each optimizer step the device status word written by bounded waits in
  the native kernels is checked, so a peer that stopped responding surfaces as
  an exception on the host instead of a hang.
"""

from __future__ import annotations

import logging
import os
import platform
import random
import secrets
import shutil
import socket
import time
from abc import ABC, abstractmethod
from dataclasses import dataclass
from os import PathLike
from pathlib import Path
from typing import Any, ClassVar, Optional, Type, Union

import numpy as np
import torch
import torch.distributed as dist

from ..config.loader import to_container
from ..config.schema import BaseEngineConfig
from ..distributed.init import initialize_process_group
from ..distributed.parallel_mesh import ParallelMesh
from ..distributed.utils import broadcast_from_main, get_local_rank, is_main_process
from ..utils.checkpointing.parallel_sl_util import load_checkpoint, save_checkpoint
from ..utils.log import init_logger, logger
from ..utils.log.backend import FileBackend, TerminalBackend, WandbBackend
from ..utils.log.timer import CudaStepTimer, Timer
from ..utils.misc import calculate_model_size, get_device, get_git_info
from ..utils.training import GradientAccumulationState, GradientScaler, accumulate_gradients, clip_grad_norm_

logging.captureWarnings(True)
logging.basicConfig(level=os.environ.get("LOGLEVEL", "ERROR").upper())


COMPLETE_MARKER = "COMPLETE"


def latest_complete_checkpoint(root: Union[str, PathLike]) -> Optional[str]:
    """Newest ``<policy>_<n>`` directory under ``root`` holding the completion marker (None if none).

    A checkpoint interrupted mid-save (or damaged afterwards and stripped of its marker) is skipped,
    so an automatic restart resumes from the last checkpoint that was fully written.
    """
    root = Path(root)
    if not root.is_dir():
        return None
    cands = [p for p in root.iterdir() if p.is_dir() and p.name.split("_")[-1].isdigit()]
    for p in sorted(cands, key=lambda p: int(p.name.split("_")[-1]), reverse=True):
        if (p / COMPLETE_MARKER).is_file():
            return str(p)
    return None


@dataclass
class TrainStepContext:
    """Mutable state for one training micro-batch."""

    data: Any
    step: int
    epoch: int
    micro_step: int
    outputs: Optional[dict[str, Any]] = None
    loss: Optional[torch.Tensor] = None
    should_sync: bool = False
    optimizer_step_completed: bool = False


def set_seed(seed: int, deterministic: bool = False) -> None:
    """Seed python, numpy and torch (all devices); optionally force deterministic kernels."""
    random.seed(seed)
    np.random.seed(seed % (2**32))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    if deterministic:
        torch.use_deterministic_algorithms(True, warn_only=True)
        os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")


class Engine(ABC):
    ConfigClass: ClassVar[Type[BaseEngineConfig]] = BaseEngineConfig
    config: BaseEngineConfig
    parallel_mesh: ParallelMesh
    model: torch.nn.Module
    optimizer: torch.optim.Optimizer
    scheduler: Any
    scaler: GradientScaler
    epoch: int = 0
    step: int = 0
    ga_state: GradientAccumulationState
    timer: Timer

    def __init__(self, config: Any):
        self.config = self.prepare_config(config)
        self.prepare_parallel()
        self.prepare_runtime_info()
        self.set_seed(self.config.seed, self.config.deterministic)
        self.prepare_logger()
        self.step_time_ms: float = 0.0
        self._cuda_timer = CudaStepTimer()
        self._step_timer_running = False

    # ------------------------------------------------------------ properties
    def prepare_config(self, config: Any) -> BaseEngineConfig:
        return self.ConfigClass.model_validate(to_container(config))

    @property
    def device(self) -> torch.device:
        return get_device(index=get_local_rank() % max(1, torch.cuda.device_count()) if torch.cuda.is_available()
                          else 0)

    @property
    def device_type(self) -> str:
        return self.device.type

    @property
    def dtype(self) -> torch.dtype:
        return {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}.get(
            self.config.optim.mixed_precision, torch.float32)

    @property
    def total_steps(self) -> int:
        if self.loop_policy == "iter":
            return self.config.loop.total_steps
        raise NotImplementedError(f"Unsupported loop policy: {self.loop_policy}")

    @property
    def project_dir(self) -> Path:
        return Path(self.config.runtime.output_dir)

    @property
    def run_id(self) -> str:
        return self.config.runtime.run_id

    @property
    def loop_policy(self) -> str:
        return self.config.loop.policy

    @property
    def _accumulate_step(self) -> int:
        return self.ga_state.micro_step

    @_accumulate_step.setter
    def _accumulate_step(self, value: int) -> None:
        self.ga_state.micro_step = int(value)

    @property
    def progress(self) -> float:
        if self.loop_policy == "iter":
            return self.step / self.total_steps
        raise ValueError(f"Unsupported loop policy: {self.loop_policy}")

    @property
    def unwrapped_model(self) -> torch.nn.Module:
        m = self.model
        while True:
            inner = getattr(m, "module", None)
            if isinstance(inner, torch.nn.Module) and inner is not m:
                m = inner
                continue
            return m

    # --------------------------------------------------------------- set-up
    def set_seed(self, seed: int, deterministic: bool = False) -> None:
        set_seed(seed, deterministic)

    def prepare_parallel(self) -> None:
        initialize_process_group()
        self.parallel_mesh = ParallelMesh.initialize(self.device.type, self.config.parallel.mesh.model_dump())

    def prepare_runtime_info(self) -> None:
        git = get_git_info()
        rt = self.config.runtime
        rt.git_info = f"<{git['branch']}> {git['commit_hash']}"
        rt.world_size = dist.get_world_size() if dist.is_initialized() else 1
        rt.hostname = socket.gethostname()
        rt.python_version = platform.python_version()
        rt.torch_version = str(torch.__version__)
        if not rt.run_id:
            local = f"{self.config.project.name}_{time.strftime('%Y%m%d%H%M%S', time.localtime())}_{secrets.token_hex(2)}"
            rt.run_id = broadcast_from_main(local)
        rt.output_dir = str(Path(self.config.project.dir) / rt.run_id)

    def prepare_logger(self) -> None:
        backends = []
        if self.config.dev_mode:
            backends = [TerminalBackend(id=self.run_id)]
        else:
            for b in self.config.log.backends:
                if b == "terminal":
                    backends.append(TerminalBackend(id=self.run_id))
                elif b == "file":
                    backends.append(FileBackend(id=self.run_id, path=Path(self.config.runtime.output_dir)))
                elif b == "wandb":
                    backends.append(WandbBackend(id=self.run_id, project=self.config.project.name,
                                                 path=Path(self.config.runtime.output_dir)))
                else:
                    raise ValueError(f"Invalid log backend: {b}")
        acc = self.config.log.accumulation_size
        init_logger(backends, interval=self.config.log.interval,
                    accumulation_size=acc if acc is not None else self.config.log.interval)

    @abstractmethod
    def prepare_model(self) -> torch.nn.Module: ...

    @abstractmethod
    def prepare_optimizer(self) -> torch.optim.Optimizer: ...

    @abstractmethod
    def prepare_scheduler(self) -> Any: ...

    @abstractmethod
    def prepare_dataloader(self, workflow: str = "train") -> Any: ...

    # ------------------------------------------------------------ checkpoint
    def save(self, force: bool = False) -> None:
        interval = self.config.checkpoint.interval
        if (not force and self.step % interval != 0) or self.config.dev_mode:
            return
        logger.info(f"Saving checkpoint for step {self.step}...")
        ckpt_root = self.project_dir / "checkpoints"
        ckpt_root.mkdir(parents=True, exist_ok=True)
        tag = f"{self.loop_policy}_{self.epoch if self.loop_policy == 'epoch' else self.step}"
        cur = ckpt_root / tag
        if is_main_process():
            existing = sorted((p for p in os.listdir(ckpt_root) if p != cur.name and p.split("_")[-1].isdigit()),
                              key=lambda p: int(p.split("_")[-1]))
            keep_existing = self.config.checkpoint.keep_n - 1
            for old in existing[: max(len(existing) - keep_existing, 0)]:
                shutil.rmtree(ckpt_root / old, ignore_errors=True)
        cur.mkdir(parents=True, exist_ok=True)
        if dist.is_initialized():
            dist.barrier()
        save_checkpoint(self.parallel_mesh.device_mesh, cur, self.model, self.optimizer, scheduler=self.scheduler,
                        scaler=self.scaler, step=self.step, epoch=self.epoch, _accumulate_step=self._accumulate_step,
                        hf_enable=self.config.checkpoint.hf_enable)
        if dist.is_initialized():
            dist.barrier()
        if is_main_process():  # written last: a checkpoint without it is incomplete and never resumed from
            (cur / COMPLETE_MARKER).write_text(str(self.step))

    def load(self, ckpt_path: Union[str, PathLike], restore_training_state: bool = True,
             restore_rng_state: bool = True) -> None:
        logger.info(f"{'Loading checkpoint' if restore_training_state else 'Initializing model from'} {ckpt_path}...")
        state = load_checkpoint(self.parallel_mesh.device_mesh, ckpt_path, self.model,
                                self.optimizer if restore_training_state else None,
                                self.scheduler if restore_training_state else None,
                                self.scaler if restore_training_state else None,
                                restore_engine_state=restore_training_state, restore_rng_state=restore_rng_state,
                                hf_enable=self.config.checkpoint.hf_enable)
        if state is None:
            return
        self.step = state["step"]
        self.epoch = state["epoch"]
        self._accumulate_step = state["_accumulate_step"]
        if hasattr(self, "timer"):
            self.timer.set_progress(self.step, self.total_steps)

    # ---------------------------------------------------------------- train
    def train(self) -> None:
        self.before_train()
        self.do_train()
        self.after_train()

    def before_train(self) -> None:
        logger.log_config(self.config.model_dump())
        logger.info("Building DataLoader...")
        self.train_loader = self.prepare_dataloader("train")
        self.evaluate_loader = self.prepare_dataloader("evaluate")
        logger.info("Building Model...")
        self.model = self.prepare_model()
        total, trainable = calculate_model_size(self.model)
        logger.info(f" - Model size: {total / 1e9:.4f} B")
        logger.info(f" - Trainable model size: {trainable / 1e9:.4f} B")
        logger.info("Building Optimizer...")
        self.optimizer = self.prepare_optimizer()
        self.ga_state = GradientAccumulationState(self.config.optim.gradient_accumulation_steps)
        logger.info("Building Scheduler...")
        self.scheduler = self.prepare_scheduler()
        logger.info("Building GradientScaler...")
        self.scaler = GradientScaler(enabled=self.dtype != torch.float32, dtype=self.dtype, device=self.device_type)
        resume = getattr(self.config, "resume", None)
        if resume == "latest":  # newest complete checkpoint of this project, if any
            resume = latest_complete_checkpoint(self.project_dir / "checkpoints")
        if resume is not None:
            self.load(resume, restore_training_state=True, restore_rng_state=True)
        from ..distributed.watchdog import start_default_watchdog

        self._watchdog = start_default_watchdog()
        logger.info("Initializing Timer...")
        self.timer = Timer(total_progress=self.total_steps, window_size=self.config.log.timer_window_size)

    def do_train(self) -> None:
        name = type(self.unwrapped_model).__name__
        logger.info(f"Start training: {name} / {type(self.optimizer).__name__} / {type(self.scheduler).__name__}...")
        self.model.train()
        self.timer.start()
        self.timer.set_progress(self.step)
        while self.progress < 1.0:
            it = iter(self.train_loader)
            try:
                while self.progress < 1.0:
                    with self.timer.scope("data_time"):
                        data = next(it)
                        ctx = TrainStepContext(data=data, step=self.step, epoch=self.epoch,
                                               micro_step=self.ga_state.micro_step)
                        prepared = self.train_pre_step(ctx)
                        if prepared is not None and prepared is not ctx:
                            ctx.data = prepared
                    if getattr(self, "_watchdog", None) is not None:
                        self._watchdog.check()  # a silent peer ends the run before the next collectives
                    with self.timer.scope("exec_time"):
                        self.train_exec_step(ctx)
                    if not ctx.optimizer_step_completed:
                        continue
                    assert ctx.outputs is not None, "The forward step must populate ctx.outputs."
                    self.step += 1
                    self.timer.tick()
                    self.train_post_step(ctx)
                    self.save()
            except StopIteration:
                self.epoch += 1
                logger.info(f"Starting epoch {self.epoch}...")

    def train_step(self, micro_batches: list[Any]) -> dict[str, Any]:
        """One optimizer step over ``micro_batches`` (host batches as the dataloader yields them):
        each goes through ``train_pre_step`` and ``train_exec_step``; the step's outputs are returned.
        This is the public single-step API the training loop, benchmarks and tests share."""
        if len(micro_batches) != int(self.config.optim.gradient_accumulation_steps):
            raise ValueError(f"expected {self.config.optim.gradient_accumulation_steps} micro-batches, "
                             f"got {len(micro_batches)}")
        ctx = None
        for data in micro_batches:
            ctx = TrainStepContext(data=data, step=self.step, epoch=self.epoch, micro_step=self.ga_state.micro_step)
            prepared = self.train_pre_step(ctx)
            if prepared is not None and prepared is not ctx:
                ctx.data = prepared
            self.train_exec_step(ctx)
        assert ctx is not None and ctx.optimizer_step_completed, "the last micro-batch must complete a step"
        self.step += 1
        return ctx.outputs or {}

    def train_pre_step(self, ctx: TrainStepContext) -> Optional[TrainStepContext]:
        return None

    def train_exec_step(self, ctx: TrainStepContext) -> None:
        if not self._step_timer_running:
            self._cuda_timer.start()
            self._step_timer_running = True
        self.forward_step(ctx)
        self.backward_step(ctx)
        self.optimizer_step(ctx)
        if ctx.optimizer_step_completed:
            self._step_timer_running = False
            self.step_time_ms = CudaStepTimer.max_over_ranks(self._cuda_timer.stop())
            self.check_device_status()

    def check_device_status(self) -> None:
        """Raise if a native kernel's bounded wait expired during the step."""
        if self.device.type != "cuda":
            return
        from ..ops import _ext

        if _ext.available():
            _ext.check_status(self.device)

    def forward_step(self, ctx: TrainStepContext) -> None:
        with torch.autocast(device_type=self.device_type, dtype=self.dtype, enabled=self.dtype != torch.float32):
            ctx.outputs = self.model(ctx.data)

    def backward_step(self, ctx: TrainStepContext) -> None:
        assert ctx.outputs is not None and "loss" in ctx.outputs and "logs" in ctx.outputs
        ctx.should_sync = self.ga_state.advance()
        ctx.loss = ctx.outputs["loss"] / self.config.optim.gradient_accumulation_steps
        with accumulate_gradients(self.model, sync=ctx.should_sync):
            self.scaler.scale(ctx.loss).backward()

    def optimizer_step(self, ctx: TrainStepContext) -> None:
        if not ctx.should_sync:
            return
        self.scaler.unscale_(self.optimizer)
        if self.config.optim.clip_grad_norm is not None:
            clip_grad_norm_(self.model, self.config.optim.clip_grad_norm)
        self.scaler.step(self.optimizer)
        self.scaler.update()
        self.scheduler.step()
        self.optimizer.zero_grad(set_to_none=True)
        ctx.optimizer_step_completed = True

    def train_post_step(self, ctx: TrainStepContext) -> None:
        logs = {"eta": self.timer.eta_string, "perf/data_time": self.timer.get_scope_time("data_time"),
                "perf/exec_time": self.timer.get_scope_time("exec_time"),
                "perf/step_time_device_ms": self.step_time_ms}
        for i, lr in enumerate(self.scheduler.get_last_lr()):
            logs[f"lr/group_{i}"] = lr
        self.last_logs = {**ctx.outputs["logs"], **logs}
        logger.log_metrics(self.last_logs, step=self.step, total_steps=self.total_steps)

    def after_train(self) -> None:
        if getattr(self, "_watchdog", None) is not None:
            self._watchdog.stop()
        self.save(force=True and not self.config.dev_mode)
        logger.info("Training finished!")
        logger.destroy()

    @torch.no_grad()
    def evaluate(self):
        raise NotImplementedError("The evaluate method must be implemented in subclasses.")
