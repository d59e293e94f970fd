"""Skill asserts: tensor parallelism.

Copy to ``recipes/<recipe>/tests/skills/tensor-parallel/asserts.py``.  With ``parallel.mesh.tensor > 1``
the native runtime shards the Qwen3 decoder Megatron-style (fused qkv / gate_up by rows, o_proj / down by
columns) and the data-parallel runtime shards what is left over the data ranks; the torch backend needs a
DTensor plan on the model and FSDP over the data ranks.  Every rank of a tensor group sees the same
tokens, so tokens and loss are counted over the data (x context) ranks only and each rank's FLOPs are
1/tp of the micro-batch's.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls


def test_config_structure(config):
    tensor = int(config_get(config, "parallel.mesh.tensor", 1))
    assert tensor >= 1
    if tensor > 1 and config_get(config, "parallel.backend_kwargs.impl", "native") == "torch":
        shard = int(config_get(config, "parallel.mesh.shard", 1))
        assert shard != 1, "the torch backend runs tensor parallelism under FSDP, not DDP (shard must be > 1)"


def test_engine_structure(engine_class):
    expect_calls(engine_class, "prepare_model", ["parallelize_model(", "parallel_mesh=", "backend_kwargs="])
    expect_calls(engine_class, "__init__", ["TokenNormedLossKit(", "dp_group="],
                 "token counts reduce over the data-parallel group, not the tensor group")
    expect_calls(engine_class, "forward_step", ["tp.world_size"], "each tensor rank reports 1/tp of the FLOPs")


def assert_before_train_end(engine):
    tp = engine.parallel_mesh.tp
    if not tp.active:
        return
    loss_group = getattr(engine.token_loss_kit, "dp_group", None)
    assert loss_group is not tp.group, "the token-loss kit must not reduce over the tensor group"
    model = engine.unwrapped_model
    heads = int(getattr(model.config, "num_attention_heads", 0))
    kv = int(getattr(model.config, "num_key_value_heads", heads))
    assert heads % tp.world_size == 0 and kv % tp.world_size == 0, (
        f"{heads} query / {kv} kv heads do not split over {tp.world_size} tensor ranks")
