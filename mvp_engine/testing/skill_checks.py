"""Building blocks for skill assert modules.

A skill's ``references/asserts.py`` is copied into ``recipes/<recipe>/tests/skills/<skill>/asserts.py``;
the recipe's structure test then calls its ``test_engine_structure(engine_class)`` /
``test_config_structure(config)`` and the smoke test wires its ``assert_<phase>_{start,end}`` hooks
around the engine's phases (:mod:`mvp_engine.testing.recipe_checks`).  The reference writes each such
module by hand around ``inspect.getsource``; here the recurring pieces are shared:

* an engine phase is checked as the source text the engine actually runs (the first definition of the
  method along the class's MRO), so a recipe that inherits a phase from a shared base is checked
  against that base;
* a requirement is a list of call sites that must appear in a phase, optionally in a given order;
* a finished optimizer step is recognised from its ``TrainStepContext`` and its logs are checked as
  finite numbers.
"""

from __future__ import annotations

import inspect
import math
import textwrap
from typing import Any, Iterable, Mapping, Optional


def phase_source(engine_class: type, name: str) -> str:
    """Dedented source of ``engine_class.<name>`` as resolved by the MRO, followed by the parents'
    definitions it delegates to through ``super().<name>(``; '' when no class defines it."""
    parts: list[str] = []
    for klass in inspect.getmro(engine_class):
        fn = klass.__dict__.get(name)
        if fn is None:
            continue
        fn = getattr(fn, "__func__", fn)
        try:
            src = textwrap.dedent(inspect.getsource(fn))
        except (OSError, TypeError):
            break
        parts.append(src)
        if f"super().{name}(" not in src:
            break
    return "\n".join(parts)


def expect_calls(engine_class: type, phase: str, needles: Iterable[str], why: str = "") -> str:
    """Every ``needle`` occurs in the phase's source; returns that source."""
    src = phase_source(engine_class, phase)
    missing = [n for n in needles if n not in src]
    assert not missing, f"{engine_class.__name__}.{phase} must contain {missing}" + (f": {why}" if why else "")
    return src


def expect_order(engine_class: type, phase: str, needles: Iterable[str], why: str = "") -> None:
    """The needles occur in the phase's source, each first occurrence after the previous one."""
    src = expect_calls(engine_class, phase, needles, why)
    positions = [src.find(n) for n in needles]
    assert positions == sorted(positions), (
        f"{engine_class.__name__}.{phase} must run {' -> '.join(needles)} in that order" + (f": {why}" if why else ""))


def config_get(config: Any, dotted: str, default: Any = None) -> Any:
    """``a.b.c`` from a dict or an attribute tree (pydantic model), ``default`` when a key is absent."""
    node = config
    for key in dotted.split("."):
        if isinstance(node, Mapping):
            if key not in node:
                return default
            node = node[key]
        elif hasattr(node, key):
            node = getattr(node, key)
        else:
            return default
    return node


def completed_step_logs(ctx: Any) -> Optional[dict]:
    """The logs of a context whose optimizer step ran (None for accumulation-only micro-steps)."""
    if not getattr(ctx, "optimizer_step_completed", False):
        return None
    outputs = getattr(ctx, "outputs", None)
    assert isinstance(outputs, dict), "a completed step's TrainStepContext.outputs must be a dict"
    logs = outputs.get("logs")
    assert isinstance(logs, dict), "a completed step must carry its logs in outputs['logs']"
    return logs


def expect_finite(logs: Mapping[str, Any], keys: Iterable[str]) -> None:
    for key in keys:
        assert key in logs, f"the step must log {key}"
        value = logs[key]
        assert isinstance(value, (int, float)) and not isinstance(value, bool), f"{key} must be a number"
        assert math.isfinite(float(value)), f"{key} must be finite (got {value})"
