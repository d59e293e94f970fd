"""Skill asserts: ring / Ulysses context parallelism.

Copy to ``recipes/<recipe>/tests/skills/context-parallel/asserts.py``.  With ``parallel.mesh.context > 1``
each rank of a context group holds two zig-zag chunks of every sequence; the host-side batch is cut
before it is copied to the device, context ranks share parameters with the data ranks (gradients and
token counts reduce over data x context), and each rank reports 1/cp of the micro-batch's FLOPs.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls, expect_order


def test_config_structure(config):
    cp = int(config_get(config, "parallel.mesh.context", 1))
    assert cp >= 1
    if cp > 1:
        assert config_get(config, "parallel.backend_kwargs.context_parallel.impl", "ring") in ("ring", "ulysses")
        seq = int(config_get(config, "data.max_seq_len", 0))
        assert seq % (2 * cp) == 0, f"max_seq_len {seq} must split into 2 x {cp} zig-zag chunks"


def test_engine_structure(engine_class):
    expect_order(engine_class, "train_pre_step", ["maybe_shard_batch(", "to_device("],
                 "cut the batch into this rank's chunks on the host, then copy")
    expect_calls(engine_class, "__init__", ["dp_cp"], "tokens and loss reduce over data x context ranks")
    expect_calls(engine_class, "forward_step", ["cp_total_tokens", "cp.world_size"])


def assert_forward_step_start(engine, ctx):
    cp = engine.parallel_mesh.cp
    if cp.active:
        assert "cp_total_tokens" in ctx.data, "a context-parallel batch records the full row length"
