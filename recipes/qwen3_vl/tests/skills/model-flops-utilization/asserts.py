"""Skill asserts: model-FLOPs utilisation with MFUKit.

Copy to ``recipes/<recipe>/tests/skills/model-flops-utilization/asserts.py``.  FLOPs are counted per
micro-batch in the forward (from the model's own formula, document-aware for packed sequences) and turned
into ``perf/mfu`` once per optimizer step from the device-timed step.
"""

from mvp_engine.testing.skill_checks import completed_step_logs, expect_calls


def test_engine_structure(engine_class):
    expect_calls(engine_class, "__init__", ["MFUKit("])
    expect_calls(engine_class, "forward_step", ["mfu_kit.accumulate_microbatch("],
                 "every micro-batch adds its FLOPs to the step's window")
    src = expect_calls(engine_class, "train_post_step", ["mfu_kit.build_log(", "step_time_seconds"])
    assert "precision" in src, "build_log needs the training precision to pick the peak"


def assert_forward_step_end(engine):
    assert engine.mfu_kit.accumulated_model_flops > 0, "a forward step must record positive model FLOPs"


def assert_train_post_step_end(engine, ctx):
    logs = completed_step_logs(ctx)
    if logs is None:
        return
    assert engine.mfu_kit.accumulated_model_flops == 0, "build_log must consume the step's FLOPs window"
    if "perf/mfu" in logs:  # absent when the device has no known peak (CPU runs)
        assert 0.0 < float(logs["perf/mfu"]) < 1.5, f"implausible MFU {logs['perf/mfu']}"
