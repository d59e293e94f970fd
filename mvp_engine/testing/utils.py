"""Test infrastructure (reference: mvp_engine/testing/utils.py:35-231), with CPU allowed.

* ``distributed_env`` sets RANK / WORLD_SIZE / LOCAL_RANK / MASTER_* for one
  worker and tears down a process group created inside it.  Unlike the
  reference it does not reject CPU: multi-rank tests run as gloo processes.
* ``spawn_workers`` runs ``fn(rank, world, port, *args)`` in ``world`` fresh
  processes and returns their results (tracebacks are re-raised in the
  parent); a per-worker timeout turns a hung rank into a failure.
* ``load_smoke_test_config`` / ``inject_engine_hook`` /
  ``load_recipe_skill_asserts`` / ``inject_engine_assert_hooks`` keep the
  reference's recipe-test contract.
* Fault-injection helpers for host-side failure tests live in
  :mod:`mvp_engine.testing.faults`.
"""

from __future__ import annotations

import importlib.util
import inspect
import multiprocessing as mp
import os
import socket
import traceback
from contextlib import contextmanager
from pathlib import Path
from types import ModuleType
from typing import Any, Callable, Optional

import torch.distributed as dist

DIST_ENV_KEYS = ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")
ENGINE_HOOK_PHASES = ("before_train", "do_train", "train_pre_step", "train_exec_step", "forward_step",
                      "backward_step", "optimizer_step", "train_post_step", "after_train")


@contextmanager
def distributed_env(*, rank: int, world_size: int, local_rank: int, master_port: int,
                    master_addr: str = "127.0.0.1"):
    prev = {k: os.environ.get(k) for k in DIST_ENV_KEYS}
    was = dist.is_initialized()
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world_size), "LOCAL_RANK": str(local_rank),
                       "MASTER_ADDR": master_addr, "MASTER_PORT": str(master_port)})
    try:
        yield
    finally:
        if not was and dist.is_initialized():
            dist.destroy_process_group()
        for k, v in prev.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def find_free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _worker(fn, rank, world, port, args, q):
    import io

    import torch

    try:
        with distributed_env(rank=rank, world_size=world, local_rank=rank, master_port=port):
            result = fn(rank, world, port, *args)
        buf = io.BytesIO()  # serialise: tensors must not travel as shared-memory handles of a dying process
        torch.save(result, buf)
        q.put((rank, "ok", buf.getvalue()))
    except BaseException:  # noqa: BLE001 - report everything to the parent
        q.put((rank, "err", traceback.format_exc()))


def spawn_workers(fn: Callable, world: int, *args: Any, timeout: float = 600.0) -> list[Any]:
    """Run ``fn(rank, world, port, *args)`` in ``world`` spawned processes; return results by rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = find_free_port()
    procs = [ctx.Process(target=_worker, args=(fn, r, world, port, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results: dict[int, Any] = {}
    errors = []
    try:
        for _ in range(world):
            rank, status, payload = q.get(timeout=timeout)
            if status == "ok":
                import io

                import torch

                results[rank] = torch.load(io.BytesIO(payload), weights_only=False)
            else:
                errors.append(f"rank {rank}:\n{payload}")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    if errors:
        raise RuntimeError("\n".join(errors))
    return [results[r] for r in range(world)]


def load_smoke_test_config(recipe_root: Path, config_name: str, *, output_dir: Path, run_id: str = "smoke",
                           config_overrides: tuple[str, ...] = (), extra_override: Optional[dict] = None) -> dict:
    """Recipe YAML <- standard smoke override <- ``extra_override`` <- dotlist (later wins)."""
    from ..config.loader import apply_dotlist, deep_merge, load_yaml

    path = Path(recipe_root) / "configs" / f"{config_name}.yaml"
    assert path.exists(), f"Config file does not exist: {path}"
    smoke = {"project": {"dir": str(output_dir)}, "runtime": {"run_id": run_id},
             "log": {"interval": 1, "backends": ["terminal", "file"]},
             "checkpoint": {"interval": 1, "keep_n": 1, "hf_enable": False}, "data": {"num_workers": 0},
             "loop": {"total_steps": 1}}
    cfg = deep_merge(load_yaml(path), smoke)
    if extra_override:
        cfg = deep_merge(cfg, extra_override)
    return apply_dotlist(cfg, list(config_overrides))


def inject_engine_hook(engine, method_name: str, *, before=None, after=None) -> None:
    original = getattr(engine, method_name)

    def wrapped(*args, **kwargs):
        if before is not None:
            before(engine, *args, **kwargs)
        result = original(*args, **kwargs)
        if after is not None:
            after(engine, result, *args, **kwargs)
        return result

    setattr(engine, method_name, wrapped)


def load_recipe_skill_asserts(recipe_root: Path) -> list[ModuleType]:
    mods = []
    for path in sorted((Path(recipe_root) / "tests" / "skills").glob("*/asserts.py")):
        name = f"{Path(recipe_root).name}_{path.parent.name.replace('-', '_')}_asserts"
        spec = importlib.util.spec_from_file_location(name, path)
        assert spec is not None and spec.loader is not None
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods.append(mod)
    return mods


def read_recipe_source(recipe_root: Path) -> str:
    skip = {".git", ".venv", "__pycache__", "pretrained", "references", "tests"}
    return "\n".join(p.read_text(encoding="utf-8") for p in sorted(Path(recipe_root).rglob("*.py"))
                     if not any(part in skip for part in p.parts))


def _call_assert(fn, payload: dict) -> None:
    params = inspect.signature(fn).parameters
    if any(p.kind == p.VAR_KEYWORD for p in params.values()):
        fn(**payload)
    else:
        fn(**{k: v for k, v in payload.items() if k in params})


def inject_engine_assert_hooks(engine: object, skill_asserts: list[ModuleType]) -> None:
    """Wrap each phase so ``assert_<phase>_start`` / ``assert_<phase>_end`` of every skill module run around it."""
    for phase in ENGINE_HOOK_PHASES:
        start, end = f"assert_{phase}_start", f"assert_{phase}_end"
        if not any(hasattr(m, start) or hasattr(m, end) for m in skill_asserts):
            continue

        def before(engine, *args, _n=start, **kwargs):
            payload = {"engine": engine, "args": args, "kwargs": kwargs}
            if args:
                payload["ctx"] = args[0]
            for m in skill_asserts:
                if hasattr(m, _n):
                    _call_assert(getattr(m, _n), payload)

        def after(engine, result, *args, _n=end, **kwargs):
            payload = {"engine": engine, "result": result, "args": args, "kwargs": kwargs}
            if args:
                payload["ctx"] = args[0]
            for m in skill_asserts:
                if hasattr(m, _n):
                    _call_assert(getattr(m, _n), payload)

        inject_engine_hook(engine, phase, before=before, after=after)
