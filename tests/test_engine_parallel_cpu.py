"""The Qwen3 recipe engine end to end on gloo ranks: tensor parallelism (with and without sequence
parallelism) and context parallelism (ring, Ulysses) -- layouts whose ranks all read the one data
stream -- reproduce the one-process loss curve over three optimizer steps: data distribution, host-side
batch cut, loss / token reductions, meta-device init of sharded weights and the optimizer included.

Data-parallel ranks read different shards of the stream, so their curves differ from one process's by
design; the runtime-level tests in ``test_fsdp_gloo.py`` feed them identical rows instead."""

from __future__ import annotations

from pathlib import Path

import pytest

from mvp_engine.testing.utils import spawn_workers

ROOT = Path(__file__).resolve().parent.parent
_TINY = ("loop.total_steps=3", "checkpoint.interval=100000", "log.backends=[terminal]",
         "model.pretrained_model_name_or_path=mvp/qwen3-tiny", "model.config_overrides.vocab_size=512",
         "model.config_overrides.num_hidden_layers=2", "optim.mixed_precision=fp32",
         "data.train_path=synthetic://text?vocab=512&min_len=16&max_len=96", "data.max_seq_len=128",
         "optim.global_batch_size=2", "model.gradient_checkpointing.enabled=false", "optim.warmup_ratio=0.0",
         "parallel.mesh.replicate=1", "parallel.mesh.shard=1")


def _run(rank, world, port, overrides, out_dir):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = ROOT / "recipes" / "qwen3"
    import_recipe_modules(root)
    cfg = load_smoke_test_config(root, "synthetic_8b", output_dir=Path(out_dir), run_id=f"r{rank}",
                                 config_overrides=_TINY + tuple(overrides))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    losses = []
    post = eng.train_post_step

    def record(ctx):
        post(ctx)
        losses.append(eng.last_logs["train/loss"])

    eng.train_post_step = record
    eng.train()
    return losses


_SINGLE: dict = {}


def _single(global_batch: int, tmp_path_factory) -> list:
    if global_batch not in _SINGLE:
        out = str(tmp_path_factory.mktemp(f"single{global_batch}"))
        _SINGLE[global_batch] = spawn_workers(_run, 1, (f"optim.global_batch_size={global_batch}",), out,
                                              timeout=600)[0]
    return _SINGLE[global_batch]


@pytest.mark.parametrize("world,overrides", [
    (2, ("parallel.mesh.tensor=2", "parallel.backend_kwargs.sequence_parallel=false")),
    (2, ("parallel.mesh.tensor=2", "parallel.backend_kwargs.sequence_parallel=true")),
    (2, ("parallel.mesh.context=2", "parallel.backend_kwargs.context_parallel.impl=ring")),
    (2, ("parallel.mesh.context=2", "parallel.backend_kwargs.context_parallel.impl=ulysses")),
], ids=["tp", "tp-sp", "cp-ring", "cp-ulysses"])
def test_engine_ranks_reproduce_one_process(world, overrides, tmp_path, tmp_path_factory):
    batch = next((int(o.split("=")[1]) for o in overrides if o.startswith("optim.global_batch_size=")), 2)
    single = _single(batch, tmp_path_factory)
    for losses in spawn_workers(_run, world, overrides, str(tmp_path), timeout=600):
        assert len(losses) == len(single) == 3
        for a, b in zip(losses, single):
            assert abs(a - b) <= 2e-5 * abs(b), (overrides, losses, single)


def _run_vl(rank, world, port, overrides, out_dir):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = ROOT / "recipes" / "qwen3_vl"
    import_recipe_modules(root)
    cfg = load_smoke_test_config(root, "synthetic_tiny", output_dir=Path(out_dir), run_id=f"v{rank}",
                                 config_overrides=("loop.total_steps=2", "checkpoint.interval=1000000",
                                                   "optim.global_batch_size=2", "optim.mixed_precision=fp32",
                                                   "parallel.mesh.shard=1") + tuple(overrides))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    losses = []
    post = eng.train_post_step

    def record(ctx):
        post(ctx)
        losses.append(eng.last_logs["train/loss"])

    eng.train_post_step = record
    eng.train()
    return losses


def test_vl_engine_tensor_parallel_reproduces_one_process(tmp_path):
    single = spawn_workers(_run_vl, 1, (), str(tmp_path / "one"), timeout=600)[0]
    for losses in spawn_workers(_run_vl, 2, ("parallel.mesh.tensor=2",), str(tmp_path / "tp"), timeout=600):
        for a, b in zip(losses, single):
            assert abs(a - b) <= 2e-5 * abs(b), (losses, single)


def test_sequence_parallel_is_refused_where_the_model_lacks_it():
    from mvp_engine.models.qwen3_vl import build_qwen3_vl
    from mvp_engine.parallel.tensor_parallel import apply_native_tensor_parallel

    model = build_qwen3_vl("mvp/qwen3-vl-tiny", device="meta")
    with pytest.raises(ValueError, match="sequence parallelism"):
        apply_native_tensor_parallel(model, sequence_parallel=True)


def _vl_with_context(rank, world, port, out_dir):
    try:
        _run_vl(rank, world, port, ("parallel.mesh.context=2",), out_dir)
    except ValueError as exc:
        return str(exc)
    return "ran"


def test_vl_engine_refuses_context_parallelism(tmp_path):
    for msg in spawn_workers(_vl_with_context, 2, str(tmp_path), timeout=300):
        assert "context parallelism" in msg
