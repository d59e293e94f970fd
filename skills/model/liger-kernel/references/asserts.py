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
    assert "cross_entropy" not in src.split(".apply(", 1)[1].split(")", 1)[0] or "exclude" in src, (
        "do not swap the cross-entropy: the token-normalised loss needs per-token losses")


def check_report(report):
    """``LigerKernelKit.apply(...)`` result: nothing excluded was applied."""
    applied = {name.rsplit(".", 1)[-1] for name in report.applied}
    assert not applied & set(report.excluded), f"excluded kernels were applied: {applied & set(report.excluded)}"
