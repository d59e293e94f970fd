"""Skill asserts: checkpoints that a crashed run can resume from.

Copy to ``recipes/<recipe>/tests/skills/failure-recovery/asserts.py``.  A checkpoint directory counts
only once its ``COMPLETE`` marker (written last, holding the optimizer step) exists; ``resume: latest``
loads the newest such directory, including the data loader's position, so the loss curve continues
where the last complete checkpoint left it.
"""

from pathlib import Path

from mvp_engine.engine.checkpoint_store import COMPLETE_MARKER, latest_complete_checkpoint
from mvp_engine.testing.skill_checks import config_get


def test_config_structure(config):
    assert int(config_get(config, "checkpoint.interval", 1)) >= 1
    assert int(config_get(config, "checkpoint.keep_n", 1)) >= 1
    resume = config_get(config, "resume")
    assert resume is None or isinstance(resume, str), "resume: unset, 'latest' or a checkpoint directory"


def assert_after_train_end(engine):
    if bool(config_get(engine.config, "dev_mode", False)):
        return  # dev runs write no checkpoints
    root = Path(engine.project_dir) / "checkpoints"
    latest = latest_complete_checkpoint(root)
    if latest is None:
        return  # nothing was due
    marker = (Path(latest) / COMPLETE_MARKER).read_text().strip()
    assert marker.lstrip("-").isdigit(), f"the completion marker of {latest} must hold the optimizer step"
    complete = [p for p in root.iterdir() if (p / COMPLETE_MARKER).is_file()]
    assert len(complete) <= int(config_get(engine.config, "checkpoint.keep_n", 1)), (
        f"{len(complete)} complete checkpoints kept, keep_n is {config_get(engine.config, 'checkpoint.keep_n')}")
