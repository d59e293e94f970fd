"""Logger + file backend: interval-gated windowed means, string metrics, message levels, and the line
format the run summariser parses."""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

from mvp_engine.utils.log import LogLevel, init_logger, logger
from mvp_engine.utils.log.backend.file import FileBackend

ROOT = Path(__file__).resolve().parent.parent


def test_file_backend_lines_and_windows(tmp_path):
    init_logger([FileBackend("run1", tmp_path)], interval=2, accumulation_size=2, level=LogLevel.INFO)
    try:
        logger.log_config({"engine": "Qwen3Engine", "optim": {"lr": 0.1}})
        for step, (loss, eta) in enumerate([(4.0, "0:00:03"), (2.0, "0:00:02"), (1.0, "0:00:01"), (5.0, "0:00:00")],
                                           start=1):
            logger.log_metrics({"train/loss": loss, "eta": eta}, step=step, total_steps=4)
        logger.debug("hidden at INFO")
        logger.warning("loss spike skipped")
    finally:
        logger.destroy()
    lines = (tmp_path / "log_run1.log").read_text().splitlines()
    metric_lines = [ln for ln in lines if "||" in ln]
    # reported every 2 updates, as the mean of the last 2 values; the ETA string goes to the header
    assert len(metric_lines) == 2
    assert "Step        2/4 ||" in metric_lines[0] and "train/loss: 3.0 |" in metric_lines[0]
    assert "ETA 0:00:02" in metric_lines[0] and "eta:" not in metric_lines[0]
    assert "train/loss: 3.0 |" in metric_lines[1] and "Step        4/4" in metric_lines[1]
    assert any("| WARN  | loss spike skipped" in ln for ln in lines)
    assert not any("hidden at INFO" in ln for ln in lines)
    assert (tmp_path / "config_run1.yaml").read_text().startswith("engine: Qwen3Engine")

    # the summariser reads the same file back
    script = ROOT / "skills" / "experiment" / "experiment-analysis" / "scripts" / "summarize_run.py"
    spec = importlib.util.spec_from_file_location("summarize_run", script)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve annotations through the module registry
    spec.loader.exec_module(mod)
    summary = mod.summarize(tmp_path, window=1)
    assert summary["metrics"]["train/loss"]["count"] == 2 and summary["health"]["finished"]
    assert summary["health"]["messages"] == {"WARN": 1} and summary["run"]["engine"] == "Qwen3Engine"


def test_timer_windows_eta_and_scopes(monkeypatch):
    """Timer arithmetic on a fake clock: per-unit tick times over a window, ETA from the remaining
    progress, named scopes, and the h:mm:ss formatting."""
    from mvp_engine.utils.log import timer as timer_mod

    now = [100.0]
    monkeypatch.setattr(timer_mod.time, "perf_counter", lambda: now[0])
    t = timer_mod.Timer(total_progress=10, window_size=2).start()
    for dt in (1.0, 3.0, 5.0):
        now[0] += dt
        t.tick()
    assert t.progress == 3 and t.progress_time == 4.0 and t.progress_time_latest == 5.0  # window of 2
    assert t.eta == 4.0 * 7 and t.eta_string == "00:00:28"
    with t.scope("data_time"):
        now[0] += 0.5
    t.record_scope("data_time", 1.5)
    assert t.get_scope_time("data_time") == 1.0 and t.get_scope_time_latest("data_time") == 1.5
    assert timer_mod.format_time(2 * 86400 + 3661) == "2d 01:01:01"


def test_cuda_step_timer_falls_back_to_host_time_on_cpu(monkeypatch):
    from mvp_engine.utils.log import timer as timer_mod

    if timer_mod.torch.cuda.is_available():
        return  # device timing is covered by the GPU runs
    now = [5.0]
    monkeypatch.setattr(timer_mod.time, "perf_counter", lambda: now[0])
    st = timer_mod.CudaStepTimer()
    st.start()
    now[0] += 0.25
    assert st.stop() == 250.0 and timer_mod.CudaStepTimer.max_over_ranks(7.0) == 7.0
