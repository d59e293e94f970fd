"""Skill asserts: sequence parallelism (on top of tensor parallelism).

Copy to ``recipes/<recipe>/tests/skills/sequence-parallel/asserts.py``.  Each tensor rank then holds
1/tp of the tokens between the tensor-parallel blocks (norms, embedding, loss), so its per-token losses
cover only its slice while its token counts cover the whole batch: the loss sum must additionally be
summed over the tensor group (``loss_sum_group``), and the weights replicated over the tensor group get
partial gradients that the runtime sums before the data-parallel reduction.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls


def test_config_structure(config):
    if config_get(config, "parallel.backend_kwargs.sequence_parallel", False):
        assert int(config_get(config, "parallel.mesh.tensor", 1)) > 1, (
            "sequence_parallel needs parallel.mesh.tensor > 1")


def test_engine_structure(engine_class):
    expect_calls(engine_class, "__init__", ["sequence_parallel", "loss_sum_group="],
                 "with sequence parallelism the loss sum also reduces over the tensor group")


def assert_before_train_end(engine):
    sp = bool(config_get(engine.config, "parallel.backend_kwargs.sequence_parallel", False))
    tp = engine.parallel_mesh.tp
    group = getattr(engine.token_loss_kit, "loss_sum_group", None)
    if sp and tp.active:
        assert group is tp.group, "sequence parallel: the token-loss kit must sum loss over the tensor group"
    else:
        assert group is None, "without sequence parallelism every rank's loss sum is already whole"
