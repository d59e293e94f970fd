"""Skill asserts: kernel swaps with LigerKernelKit.

Copy to ``recipes/<recipe>/tests/skills/liger-kernel/asserts.py``.  The engine's own models already run
sm_100a kernels, so the kit's ``official`` route has nothing to patch; the ``custom`` route rebinds
``module.attr`` of third-party model code (for example to an ``mvp_engine.ops`` function).  A swap only
affects models built after it, and cross-entropy swaps stay excluded: the token-normalised loss needs
per-token losses, which a fused mean-reducing loss would not return.
"""

from mvp_engine.testing.skill_checks import phase_source


def test_engine_structure(engine_class):
    src = phase_source(engine_class, "prepare_model")
    if "LigerKernelKit" not in src and "liger_kernel_kit" not in src:
        return  # the recipe does not swap kernels
    build = src.find("build_model(")
    apply = src.find(".apply(")
    assert apply >= 0, "LigerKernelKit.apply must be called"
    assert build < 0 or apply < build, "swap kernels before the model is built"
    call = src.split(".apply(", 1)[1].split(")", 1)[0]
    assert "excluded_modules=()" not in call.replace(" ", ""), (
        "keep the loss kernels excluded: the token-normalised loss needs per-token losses")


def check_report(report, excluded=("cross_entropy", "fused_linear_cross_entropy")):
    """``LigerKernelKit.apply(...)`` result: no excluded kernel was switched on, and on the custom route
    every enabled kernel rebound exactly one symbol."""
    enabled = {name for name, on in (report.applied or {}).items() if on}
    assert not enabled & set(excluded), f"excluded kernels were applied: {sorted(enabled & set(excluded))}"
    if report.route == "custom":
        assert len(report.patched) == len(enabled), (report.patched, enabled)
