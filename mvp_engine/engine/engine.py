"""Template-method training engine.

Public contract (the reference's, ``mvp_engine/engine/engine.py:50-592`` there): recipes
subclass :class:`Engine`, implement ``prepare_model / prepare_optimizer /
prepare_scheduler / prepare_dataloader`` and may override any hook below::

    __init__  : prepare_config -> prepare_parallel -> prepare_runtime_info
                -> set_seed -> prepare_logger
    train()   : before_train -> do_train -> after_train
    do_train  : per micro-batch  train_pre_step -> train_exec_step
                (forward_step -> backward_step -> optimizer_step);
                after each optimizer step  train_post_step -> save

How this engine runs that contract:

* the micro-batch stream (:meth:`_micro_batches`) is one generator that rolls
  over epochs; the loop in :meth:`do_train` and the public single-step API
  :meth:`train_step` stage batches through the same :meth:`_stage` helper;
* every optimizer step is timed on the device with CUDA events
  (``self.step_time_ms``, max over ranks) next to the host ``Timer``;
* after each optimizer step the device status word that the native kernels'
  bounded waits write is checked, so a peer that stopped answering becomes a host
  exception instead of a hang; a store heartbeat watchdog is polled before each
  micro-batch;
* checkpoint directories are committed with a completion marker and pruned only
  after the new one is complete (:class:`~.checkpoint_store.CheckpointStore`);
  ``resume: latest`` picks the newest complete one.  The data loader's position
  travels in the per-rank engine state when the loader can report it.
"""

from __future__ import annotations

import logging
import os
import platform
import random
import secrets
import socket
import time
from abc import ABC, abstractmethod
from dataclasses import dataclass
from os import PathLike
from pathlib import Path
from typing import Any, Callable, ClassVar, Iterator, Optional, Type, Union

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
from ..utils.tracing import StepTracer, TraceConfig
from ..utils.training import GradientAccumulationState, GradientScaler, accumulate_gradients, clip_grad_norm_
from .checkpoint_store import COMPLETE_MARKER, CheckpointStore, latest_complete_checkpoint

logging.captureWarnings(True)
logging.basicConfig(level=os.environ.get("LOGLEVEL", "ERROR").upper())

__all__ = ["COMPLETE_MARKER", "Engine", "TrainStepContext", "latest_complete_checkpoint", "set_seed"]

_COMPUTE_DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


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
    """Seed python, numpy and torch (every device); optionally ask for deterministic kernels."""
    random.seed(seed)
    np.random.seed(seed % (2**32))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    if deterministic:
        os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")
        torch.use_deterministic_algorithms(True, warn_only=True)


def _log_backend_factories(engine: "Engine") -> dict[str, Callable[[], Any]]:
    out_dir = Path(engine.config.runtime.output_dir)
    return {
        "terminal": lambda: TerminalBackend(id=engine.run_id),
        "file": lambda: FileBackend(id=engine.run_id, path=out_dir),
        "wandb": lambda: WandbBackend(id=engine.run_id, project=engine.config.project.name, path=out_dir),
    }


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
        self._watchdog = None
        # phase ranges only (MVP_NVTX=1 or trace.nvtx) until before_train builds the configured tracer
        self.tracer = StepTracer(TraceConfig(nvtx=self.config.trace.nvtx))

    # ------------------------------------------------------------ properties
    def prepare_config(self, config: Any) -> BaseEngineConfig:
        return self.ConfigClass.model_validate(to_container(config))

    @property
    def device(self) -> torch.device:
        if not torch.cuda.is_available():
            return get_device(index=0)
        return get_device(index=get_local_rank() % max(1, torch.cuda.device_count()))

    @property
    def device_type(self) -> str:
        return self.device.type

    @property
    def dtype(self) -> torch.dtype:
        return _COMPUTE_DTYPES.get(self.config.optim.mixed_precision, torch.float32)

    @property
    def loop_policy(self) -> str:
        return self.config.loop.policy

    def _require_iter_policy(self, what: str, exc: type) -> None:
        if self.loop_policy != "iter":
            raise exc(f"Unsupported loop policy for {what}: {self.loop_policy}")

    @property
    def total_steps(self) -> int:
        self._require_iter_policy("total_steps", NotImplementedError)
        return self.config.loop.total_steps

    @property
    def progress(self) -> float:
        self._require_iter_policy("progress", ValueError)
        return self.step / self.total_steps

    @property
    def project_dir(self) -> Path:
        return Path(self.config.runtime.output_dir)

    @property
    def run_id(self) -> str:
        return self.config.runtime.run_id

    @property
    def _accumulate_step(self) -> int:
        return self.ga_state.micro_step

    @_accumulate_step.setter
    def _accumulate_step(self, value: int) -> None:
        self.ga_state.micro_step = int(value)

    @property
    def unwrapped_model(self) -> torch.nn.Module:
        """The innermost module under DDP-style ``.module`` wrappers."""
        m = self.model
        while isinstance(getattr(m, "module", None), torch.nn.Module) and m.module is not m:
            m = m.module
        return m

    # --------------------------------------------------------------- set-up
    def set_seed(self, seed: int, deterministic: bool = False) -> None:
        set_seed(seed, deterministic)

    def prepare_parallel(self) -> None:
        initialize_process_group()
        self.parallel_mesh = ParallelMesh.initialize(self.device.type, self.config.parallel.mesh.model_dump())

    def prepare_runtime_info(self) -> None:
        rt = self.config.runtime
        git = get_git_info()
        rt.git_info = f"<{git['branch']}> {git['commit_hash']}"
        rt.world_size = dist.get_world_size() if dist.is_initialized() else 1
        rt.hostname = socket.gethostname()
        rt.python_version = platform.python_version()
        rt.torch_version = str(torch.__version__)
        if not rt.run_id:
            stamp = time.strftime("%Y%m%d%H%M%S", time.localtime())
            rt.run_id = broadcast_from_main(f"{self.config.project.name}_{stamp}_{secrets.token_hex(2)}")
        rt.output_dir = str(Path(self.config.project.dir) / rt.run_id)

    def prepare_logger(self) -> None:
        factories = _log_backend_factories(self)
        names = ["terminal"] if self.config.dev_mode else list(self.config.log.backends)
        unknown = [n for n in names if n not in factories]
        if unknown:
            raise ValueError(f"Invalid log backend: {unknown[0]}")
        acc = self.config.log.accumulation_size
        init_logger([factories[n]() for n in names], interval=self.config.log.interval,
                    accumulation_size=self.config.log.interval if acc is None else acc)

    @abstractmethod
    def prepare_model(self) -> torch.nn.Module: ...

    @abstractmethod
    def prepare_optimizer(self) -> torch.optim.Optimizer: ...

    @abstractmethod
    def prepare_scheduler(self) -> Any: ...

    @abstractmethod
    def prepare_dataloader(self, workflow: str = "train") -> Any: ...

    # ------------------------------------------------------------ checkpoint
    def _checkpoint_store(self) -> CheckpointStore:
        return CheckpointStore(self.project_dir / "checkpoints", self.config.checkpoint.keep_n,
                               is_writer=is_main_process())

    def _checkpoint_tag(self) -> str:
        counter = self.epoch if self.loop_policy == "epoch" else self.step
        return f"{self.loop_policy}_{counter}"

    def _data_state(self) -> Optional[dict]:
        loader = getattr(self, "train_loader", None)
        getter = getattr(loader, "state_dict", None)
        return getter() if callable(getter) else None

    def _data_coord(self) -> tuple[int, int]:
        """(rank, size) of this rank's share of the data stream: ranks of one data-parallel coordinate
        (tensor and context ranks) read the same stream."""
        dp = self.parallel_mesh.dp
        return int(dp.rank), int(dp.world_size)

    def save(self, force: bool = False) -> None:
        due = force or self.step % self.config.checkpoint.interval == 0
        if self.config.dev_mode or not due:
            return
        store, tag = self._checkpoint_store(), self._checkpoint_tag()
        # rank 0's view of the file system decides, so every rank takes the same branch (and barriers)
        if broadcast_from_main(store.is_current(tag, self.step)):
            logger.info(f"Checkpoint {tag} already holds step {self.step}; not rewritten.")
            return
        logger.info(f"Saving checkpoint for step {self.step}...")
        target = store.begin(tag)
        save_checkpoint(self.parallel_mesh.device_mesh, target, self.model, self.optimizer, scheduler=self.scheduler,
                        scaler=self.scaler, step=self.step, epoch=self.epoch, _accumulate_step=self._accumulate_step,
                        hf_enable=self.config.checkpoint.hf_enable, data_state=self._data_state(),
                        data_coord=self._data_coord())
        store.commit(tag, self.step)

    def load(self, ckpt_path: Union[str, PathLike], restore_training_state: bool = True,
             restore_rng_state: bool = True) -> None:
        verb = "Loading checkpoint" if restore_training_state else "Initializing model from"
        logger.info(f"{verb} {ckpt_path}...")
        restore = restore_training_state
        state = load_checkpoint(self.parallel_mesh.device_mesh, ckpt_path, self.model,
                                optimizer=self.optimizer if restore else None,
                                scheduler=self.scheduler if restore else None,
                                scaler=self.scaler if restore else None,
                                restore_engine_state=restore, restore_rng_state=restore_rng_state,
                                hf_enable=self.config.checkpoint.hf_enable, data_coord=self._data_coord())
        if state is None:
            return
        self.step, self.epoch = int(state["step"]), int(state["epoch"])
        self._accumulate_step = state["_accumulate_step"]
        data_state = state.get("data_state")
        loader = getattr(self, "train_loader", None)
        if data_state is not None and callable(getattr(loader, "load_state_dict", None)):
            loader.load_state_dict(data_state)
        if hasattr(self, "timer"):
            self.timer.set_progress(self.step, self.total_steps)

    # ---------------------------------------------------------------- train
    def train(self) -> None:
        self.before_train()
        self.do_train()
        self.after_train()

    def _build_loaders(self) -> None:
        self.train_loader = self.prepare_dataloader("train")
        self.evaluate_loader = self.prepare_dataloader("evaluate")

    def _build_model(self) -> None:
        self.model = self.prepare_model()
        total, trainable = calculate_model_size(self.model)
        logger.info(f" - Model size: {total / 1e9:.4f} B")
        logger.info(f" - Trainable model size: {trainable / 1e9:.4f} B")

    def _build_optimizer(self) -> None:
        self.optimizer = self.prepare_optimizer()
        self.ga_state = GradientAccumulationState(self.config.optim.gradient_accumulation_steps)

    def _build_scheduler(self) -> None:
        self.scheduler = self.prepare_scheduler()

    def _build_scaler(self) -> None:
        self.scaler = GradientScaler(enabled=self.dtype != torch.float32, dtype=self.dtype, device=self.device_type)

    def _resume_source(self) -> Optional[str]:
        resume = getattr(self.config, "resume", None)
        if resume == "latest":  # the newest complete checkpoint of this run (rank 0's view), if there is one
            return broadcast_from_main(latest_complete_checkpoint(self.project_dir / "checkpoints"))
        return resume

    def before_train(self) -> None:
        logger.log_config(self.config.model_dump())
        for label, build in (("DataLoader", self._build_loaders), ("Model", self._build_model),
                             ("Optimizer", self._build_optimizer), ("Scheduler", self._build_scheduler),
                             ("GradientScaler", self._build_scaler)):
            logger.info(f"Building {label}...")
            build()
        source = self._resume_source()
        if source is not None:
            self.load(source, restore_training_state=True, restore_rng_state=True)
        from ..distributed.watchdog import start_default_watchdog

        self._watchdog = start_default_watchdog()
        rank = dist.get_rank() if dist.is_available() and dist.is_initialized() else 0
        self.tracer.close()
        self.tracer = StepTracer(self.config.trace, out_dir=self.project_dir / "profile", rank=rank)
        hooked = self.tracer.attach_blocks(self.unwrapped_model)
        if hooked:
            logger.info(f"NVTX ranges on {hooked} blocks")
        logger.info("Initializing Timer...")
        self.timer = Timer(total_progress=self.total_steps, window_size=self.config.log.timer_window_size)

    def _micro_batches(self) -> Iterator[Any]:
        """Endless stream of training batches; each pass over the loader is one epoch."""
        while True:
            empty = True
            for batch in self.train_loader:
                empty = False
                yield batch
            if empty:
                raise RuntimeError("the training data loader produced no batches")
            self.epoch += 1
            logger.info(f"Starting epoch {self.epoch}...")

    def _stage(self, data: Any) -> TrainStepContext:
        """Wrap one host batch in a step context and run ``train_pre_step`` on it."""
        ctx = TrainStepContext(data=data, step=self.step, epoch=self.epoch, micro_step=self.ga_state.micro_step)
        prepared = self.train_pre_step(ctx)
        if prepared is not None and prepared is not ctx:
            ctx.data = prepared
        return ctx

    def do_train(self) -> None:
        parts = [type(self.unwrapped_model).__name__, type(self.optimizer).__name__, type(self.scheduler).__name__]
        logger.info(f"Start training: {' / '.join(parts)}...")
        self.model.train()
        self.timer.start()
        self.timer.set_progress(self.step)
        stream = self._micro_batches()
        while self.progress < 1.0:
            self.tracer.begin_step(self.step)
            with self.timer.scope("data_time"), self.tracer.range("data"):
                ctx = self._stage(next(stream))
            if self._watchdog is not None:
                self._watchdog.check()  # a silent peer ends the run before the next collective
            with self.timer.scope("exec_time"):
                self.train_exec_step(ctx)
            if ctx.optimizer_step_completed:
                assert ctx.outputs is not None, "The forward step must populate ctx.outputs."
                self.tracer.end_step(self.step)
                self.step += 1
                self.timer.tick()
                self.train_post_step(ctx)
                self.save()

    def train_step(self, micro_batches: list[Any]) -> dict[str, Any]:
        """One optimizer step over ``micro_batches`` (host batches, as the data loader yields them).

        Each batch is staged through ``train_pre_step`` and run through ``train_exec_step``; the last
        one must complete the optimizer step.  Returns that step's outputs.  The benchmark and the
        tests drive training through this call."""
        expected = int(self.config.optim.gradient_accumulation_steps)
        if len(micro_batches) != expected:
            raise ValueError(f"expected {expected} micro-batches, got {len(micro_batches)}")
        contexts = []
        self.tracer.begin_step(self.step)
        for data in micro_batches:
            with self.tracer.range("data"):
                ctx = self._stage(data)
            self.train_exec_step(ctx)
            contexts.append(ctx)
        if not contexts[-1].optimizer_step_completed:
            raise RuntimeError("the last micro-batch did not complete an optimizer step")
        self.tracer.end_step(self.step)
        self.step += 1
        return contexts[-1].outputs or {}

    def train_pre_step(self, ctx: TrainStepContext) -> Optional[TrainStepContext]:
        return None

    def train_exec_step(self, ctx: TrainStepContext) -> None:
        if not self._step_timer_running:
            self._cuda_timer.start()
            self._step_timer_running = True
        with self.tracer.range("forward"):
            self.forward_step(ctx)
        with self.tracer.range("backward"):
            self.backward_step(ctx)
        with self.tracer.range("optimizer"):
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
        mixed = self.dtype != torch.float32
        with torch.autocast(device_type=self.device_type, dtype=self.dtype, enabled=mixed):
            ctx.outputs = self.model(ctx.data)

    def backward_step(self, ctx: TrainStepContext) -> None:
        out = ctx.outputs
        missing = [k for k in ("loss", "logs") if out is None or k not in out]
        assert not missing, f"the model output lacks {missing}"
        ctx.should_sync = self.ga_state.advance()
        ctx.loss = out["loss"] / self.config.optim.gradient_accumulation_steps
        with accumulate_gradients(self.model, sync=ctx.should_sync):
            self.scaler.scale(ctx.loss).backward()

    def _apply_update(self) -> None:
        """Unscale, clip, step, advance the schedule and clear gradients."""
        self.scaler.unscale_(self.optimizer)
        limit = self.config.optim.clip_grad_norm
        if limit is not None:
            clip_grad_norm_(self.model, limit)
        self.scaler.step(self.optimizer)
        self.scaler.update()
        self.scheduler.step()
        self.optimizer.zero_grad(set_to_none=True)

    def optimizer_step(self, ctx: TrainStepContext) -> None:
        if ctx.should_sync:
            self._apply_update()
            ctx.optimizer_step_completed = True

    def train_post_step(self, ctx: TrainStepContext) -> None:
        logs = dict(ctx.outputs["logs"])
        logs.update({"eta": self.timer.eta_string, "perf/data_time": self.timer.get_scope_time("data_time"),
                     "perf/exec_time": self.timer.get_scope_time("exec_time"),
                     "perf/step_time_device_ms": self.step_time_ms})
        logs.update({f"lr/group_{i}": lr for i, lr in enumerate(self.scheduler.get_last_lr())})
        self.last_logs = logs
        logger.log_metrics(logs, step=self.step, total_steps=self.total_steps)

    def after_train(self) -> None:
        if self._watchdog is not None:
            self._watchdog.stop()
        self.tracer.close()
        if not self.config.dev_mode:
            self.save(force=True)
        logger.info("Training finished!")
        logger.destroy()

    @torch.no_grad()
    def evaluate(self):
        raise NotImplementedError("The evaluate method must be implemented in subclasses.")
