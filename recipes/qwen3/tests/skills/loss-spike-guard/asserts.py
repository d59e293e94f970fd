"""Skill asserts: skipping loss spikes with the token-loss kit's guard.

Copy to ``recipes/<recipe>/tests/skills/loss-spike-guard/asserts.py``.  The guard compares each
micro-batch's mean token loss (reduced over the data-parallel group, so every rank decides alike) with
the running window; a spike contributes a zero loss, so backward still runs on every rank and the
collectives stay matched.
"""

from mvp_engine.testing.skill_checks import config_get, expect_calls, expect_order


def test_config_structure(config):
    mult = config_get(config, "optim.loss_spike_skip_multiplier")
    assert mult is None or float(mult) > 0, "loss_spike_skip_multiplier is unset (off) or positive"
    assert int(config_get(config, "optim.loss_spike_skip_window_size", 1)) >= 1
    assert int(config_get(config, "optim.loss_spike_skip_min_history", 1)) >= 1


def test_engine_structure(engine_class):
    expect_calls(engine_class, "__init__",
                 ["build_loss_guard(", "loss_spike_skip_multiplier", "loss_spike_skip_window_size",
                  "loss_spike_skip_min_history"], "the guard is built once, from the optimizer config")
    # decide before recording the micro-batch; a skipped batch still runs backward (zero loss)
    expect_order(engine_class, "backward_step", ["guard_loss(", "accumulate_microbatch(", ".backward()"])
    src = expect_calls(engine_class, "backward_step", ["* 0.0"], "a skipped micro-batch backpropagates zero")
    assert "return" not in src.split("guard_loss(", 1)[1].split("accumulate_microbatch(", 1)[0], (
        "a skipped micro-batch must not leave backward_step early: the other ranks' collectives would hang")


def assert_backward_step_end(engine, ctx):
    kit = getattr(engine, "token_loss_kit", None)
    guard = getattr(kit, "loss_guard", None)
    assert guard is not None, "the engine must keep the guard on its token-loss kit"
    assert ctx.loss is not None, "backward_step must set ctx.loss (the backpropagated loss)"
