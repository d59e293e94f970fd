"""Failure detection on host ranks (gloo / store / files): nothing here touches a GPU.

* a rank that exits without warning is reported by the heartbeat watchdog of the survivors;
* a collective whose peer never joins ends with an error at the process-group timeout;
* a store key that is dropped makes its waiter time out instead of blocking;
* a checkpoint whose save was interrupted (or damaged) is skipped by ``resume: latest``.
"""

import multiprocessing as mp
import os
import time
from pathlib import Path

import pytest
import torch

from mvp_engine.testing.utils import find_free_port


def _watch_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), MVP_PG_TIMEOUT_S="20")
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.distributed.watchdog import HeartbeatWatchdog, PeerFailureError
    from mvp_engine.testing.faults import exit_abruptly
    from torch.distributed.distributed_c10d import _get_default_store

    initialize_process_group()
    wd = HeartbeatWatchdog(_get_default_store(), rank, world, interval_s=0.2, timeout_s=1.5).start()
    dist.barrier()
    if rank == world - 1:
        time.sleep(0.5)
        exit_abruptly()
    t0 = time.monotonic()
    while time.monotonic() - t0 < 15:
        try:
            wd.check()
        except PeerFailureError as e:
            q.put((rank, e.ranks, round(time.monotonic() - t0, 2)))
            wd.stop()
            return
        time.sleep(0.1)
    q.put((rank, [], None))


def test_heartbeat_reports_a_rank_that_exits():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = find_free_port()
    world = 3
    procs = [ctx.Process(target=_watch_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=60) for _ in range(world - 1)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert procs[-1].exitcode == 17
    for rank, failed, dt in got:
        assert failed == [world - 1], (rank, failed)
        assert dt is not None and dt < 10


def _timeout_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), MVP_PG_TIMEOUT_S="3")
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group

    initialize_process_group()
    dist.barrier()
    if rank == 1:
        time.sleep(12)  # never joins the collective below in time
        q.put((rank, "slept", None))
        return
    t0 = time.monotonic()
    try:
        x = torch.ones(4)
        dist.all_reduce(x)
        q.put((rank, "completed", None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__, round(time.monotonic() - t0, 2)))


def test_collective_with_a_missing_peer_ends_at_the_pg_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = find_free_port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (what, dt) for r, what, dt in (q.get(timeout=60) for _ in range(2))}
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    what, dt = res[0]
    assert what != "completed" and dt is not None and dt < 11


def test_dropped_store_key_times_out():
    from datetime import timedelta

    from torch.distributed import TCPStore

    from mvp_engine.testing.faults import drop_store_key

    store = TCPStore("127.0.0.1", find_free_port(), 1, True, timeout=timedelta(seconds=2))
    store.set("ready/0", "1")
    assert drop_store_key(store, "ready/0")
    t0 = time.monotonic()
    with pytest.raises(Exception):
        store.wait(["ready/0"], timedelta(seconds=1))
    assert time.monotonic() - t0 < 5


def test_resume_latest_skips_incomplete_checkpoints(tmp_path):
    from mvp_engine.engine.engine import COMPLETE_MARKER, latest_complete_checkpoint
    from mvp_engine.testing.faults import corrupt_file, remove_completion_marker

    root = tmp_path / "checkpoints"
    for step in (10, 20, 30):
        d = root / f"iter_{step}"
        (d / "model").mkdir(parents=True)
        (d / "model" / "shard.bin").write_bytes(os.urandom(64))
        (d / COMPLETE_MARKER).write_text(str(step))
    assert latest_complete_checkpoint(root) == str(root / "iter_30")
    corrupt_file(root / "iter_30" / "model" / "shard.bin")
    remove_completion_marker(root / "iter_30")  # a torn save never gets its marker
    assert latest_complete_checkpoint(root) == str(root / "iter_20")
    (root / "iter_40").mkdir()  # interrupted before anything was written
    assert latest_complete_checkpoint(root) == str(root / "iter_20")
    assert latest_complete_checkpoint(tmp_path / "none") is None


def _resume_run(rank, world, port, out_dir, steps, resume):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = Path(__file__).resolve().parent.parent / "recipes" / "magic_transformer"
    import_recipe_modules(root)
    over = [f"loop.total_steps={steps}", "checkpoint.interval=2", "checkpoint.keep_n=5", "log.interval=1",
            "log.backends=[terminal]"]
    if resume:
        over.append("resume=latest")
    cfg = load_smoke_test_config(root, "train", output_dir=Path(out_dir), run_id="fixed-run",
                                 config_overrides=tuple(over))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    eng.before_train()
    start = eng.step
    eng.do_train()
    eng.after_train()
    return start, eng.step


def test_engine_resumes_from_latest_complete_checkpoint(tmp_path):
    from mvp_engine.testing import spawn_workers

    first = spawn_workers(_resume_run, 1, str(tmp_path), 4, False, timeout=300)[0]
    assert first == (0, 4)
    ckpts = sorted(p.name for p in (tmp_path / "fixed-run" / "checkpoints").iterdir())
    assert "iter_4" in ckpts
    second = spawn_workers(_resume_run, 1, str(tmp_path), 6, True, timeout=300)[0]
    assert second == (4, 6)


def _fake_ckpt(store, tag, step, *, interrupt=False):
    path = store.begin(tag)
    (path / "model").mkdir(exist_ok=True)
    (path / "model" / "shard.bin").write_bytes(os.urandom(32))
    if interrupt:
        raise RuntimeError("killed mid-save")
    store.commit(tag, step)


def test_checkpoint_rewrite_interrupted_is_not_resumed(tmp_path):
    """A directory being rewritten loses its marker first, so a crash mid-rewrite falls back to the
    previous complete checkpoint; a save of a step that is already complete is recognised."""
    from mvp_engine.engine.checkpoint_store import CheckpointStore, latest_complete_checkpoint

    root = tmp_path / "checkpoints"
    store = CheckpointStore(root, keep_n=3, is_writer=True, barrier=lambda: None)
    _fake_ckpt(store, "epoch_1", 10)
    _fake_ckpt(store, "epoch_2", 20)
    assert store.is_current("epoch_2", 20) and not store.is_current("epoch_2", 25)
    assert latest_complete_checkpoint(root) == str(root / "epoch_2")
    with pytest.raises(RuntimeError):
        _fake_ckpt(store, "epoch_2", 25, interrupt=True)  # same tag, new step, dies half way
    assert latest_complete_checkpoint(root) == str(root / "epoch_1")


def test_checkpoint_retention_counts_complete_only(tmp_path):
    from mvp_engine.engine.checkpoint_store import CheckpointStore, latest_complete_checkpoint

    root = tmp_path / "checkpoints"
    store = CheckpointStore(root, keep_n=1, is_writer=True, barrier=lambda: None)
    _fake_ckpt(store, "iter_2", 2)
    with pytest.raises(RuntimeError):
        _fake_ckpt(store, "iter_4", 4, interrupt=True)
    # keep_n=1 and a failed save: the complete checkpoint survives, the partial one is not resumable
    assert latest_complete_checkpoint(root) == str(root / "iter_2")
    _fake_ckpt(store, "iter_6", 6)
    names = sorted(p.name for p in root.iterdir())
    assert names == ["iter_6"], names  # older complete one pruned after the new marker; stale partial gone


class _FlakyStore:
    """A store whose round trips fail while ``down`` is set (a transient TCPStore timeout)."""

    def __init__(self):
        self.kv, self.down = {}, False

    def _guard(self):
        if self.down:
            raise TimeoutError("store timeout")

    def set(self, k, v):
        self._guard()
        self.kv[k] = v.encode() if isinstance(v, str) else v

    def get(self, k):
        self._guard()
        return self.kv[k]

    def check(self, keys):
        self._guard()
        return all(k in self.kv for k in keys)


def test_watchdog_survives_a_transient_store_error():
    from mvp_engine.distributed.watchdog import HeartbeatWatchdog, PeerFailureError

    store = _FlakyStore()
    peer = HeartbeatWatchdog(store, 1, 2, interval_s=0.05, timeout_s=0.6)
    me = HeartbeatWatchdog(store, 0, 2, interval_s=0.05, timeout_s=0.6).start()
    peer.start()
    try:
        time.sleep(0.2)
        store.down = True  # one short outage, well under the timeout
        time.sleep(0.2)
        store.down = False
        time.sleep(0.3)
        me.check()  # no peer marked failed
        store.down = True  # an outage longer than the timeout does end the run
        time.sleep(1.0)
        with pytest.raises(PeerFailureError):
            me.check()
    finally:
        store.down = False
        me.stop()
        peer.stop()


class _Crash(RuntimeError):
    pass


def _continuity_run(rank, world, port, out_dir, steps, resume, crash_at=None):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = Path(__file__).resolve().parent.parent / "recipes" / "qwen3"
    import_recipe_modules(root)
    over = [f"loop.total_steps={steps}", "checkpoint.interval=2", "checkpoint.keep_n=5", "log.backends=[terminal]",
            "model.pretrained_model_name_or_path=mvp/qwen3-tiny", "model.config_overrides.vocab_size=512",
            "model.config_overrides.num_hidden_layers=2", "optim.mixed_precision=fp32",
            "data.train_path=synthetic://text?vocab=512&min_len=16&max_len=96", "data.max_seq_len=128",
            "optim.global_batch_size=2", "model.gradient_checkpointing.enabled=false"]
    if resume:
        over.append("resume=latest")
    cfg = load_smoke_test_config(root, "synthetic_8b", output_dir=Path(out_dir), run_id="cont",
                                 config_overrides=tuple(over))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    losses = {}
    real_post = eng.train_post_step

    def record(ctx):
        real_post(ctx)
        losses[eng.step] = float(eng.last_logs["train/loss"])
        if crash_at is not None and eng.step == crash_at:
            raise _Crash  # the process "dies" after this step's update, before its checkpoint

    eng.train_post_step = record
    eng.before_train()
    try:
        eng.do_train()
    except _Crash:
        return losses
    eng.after_train()
    return losses


def test_resume_continues_the_loss_curve(tmp_path):
    """A run that dies during step 3 of 4 resumes from its step-2 checkpoint: steps 3 and 4 reproduce the
    uninterrupted run (model, optimizer, scheduler, RNG and the data loader's position all come back)."""
    from mvp_engine.testing import spawn_workers

    straight = spawn_workers(_continuity_run, 1, str(tmp_path / "a"), 4, False, timeout=600)[0]
    first = spawn_workers(_continuity_run, 1, str(tmp_path / "b"), 4, False, 3, timeout=600)[0]  # dies in step 3
    resumed = spawn_workers(_continuity_run, 1, str(tmp_path / "b"), 4, True, timeout=600)[0]
    assert sorted(resumed) == [3, 4], resumed
    for step in (1, 2):
        assert abs(first[step] - straight[step]) < 1e-6, (first, straight)
    for step in (3, 4):
        assert abs(resumed[step] - straight[step]) < 1e-5 * abs(straight[step]), (resumed, straight)
