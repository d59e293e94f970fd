"""Skill asserts: token-normalised loss with TokenNormedLossKit.

Copy to ``recipes/<recipe>/tests/skills/token-normalized-loss/asserts.py``.  The structure check reads
the engine's phase methods; the runtime check looks at every completed optimizer step of a smoke run.
"""

from mvp_engine.testing.skill_checks import completed_step_logs, expect_calls, expect_finite, expect_order


def test_engine_structure(engine_class):
    expect_calls(engine_class, "__init__", ["TokenNormedLossKit("], "the engine owns one token-loss kit")
    expect_calls(engine_class, "prepare_model", ["apply_chunked_token_loss_patch"],
                 "the model must return one loss per token, not a mean")
    expect_calls(engine_class, "backward_step",
                 [".sum()", "accumulate_microbatch(", "effective_tokens", "total_tokens", "backward_divisor"],
                 "each micro-batch backpropagates its loss sum over a divisor fixed for the whole step")
    # the window is reduced across ranks before the gradients are touched; the rescale happens on
    # unscaled gradients and before clipping, so the clip sees the gradient of the mean token loss
    expect_order(engine_class, "optimizer_step",
                 ["reduce_window(", "unscale_(", "rescale_gradients(", "clip_grad_norm_(", ".step("])
    expect_calls(engine_class, "optimizer_step", ["token_loss_kit.reset()"], "the next step starts a new window")
    expect_calls(engine_class, "train_post_step", ["tokens/total", "tokens/effective", "perf/toks_per_sec"])


def assert_train_post_step_end(engine, ctx):
    logs = completed_step_logs(ctx)
    if logs is None:
        return
    expect_finite(logs, ("train/loss", "tokens/total", "tokens/effective", "perf/toks_per_sec"))
    eff, tot = int(logs["tokens/effective"]), int(logs["tokens/total"])
    assert 0 < eff <= tot, f"supervised tokens must be positive and at most the step's tokens ({eff} / {tot})"
    out = ctx.outputs
    if "global_loss_sum" in out:  # train/loss is the mean over the step's supervised tokens of all ranks
        mean = float(out["global_loss_sum"]) / eff
        assert abs(float(logs["train/loss"]) - mean) <= 1e-6 * max(1.0, abs(mean)), (logs["train/loss"], mean)
