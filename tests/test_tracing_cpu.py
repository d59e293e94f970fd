"""Step tracing: the disabled tracer is a shared no-op, NVTX block hooks attach and detach, and a
training run with a profiler window writes a Chrome trace holding the engine's phase labels."""

from __future__ import annotations

import json
from pathlib import Path

import torch

from mvp_engine.testing.utils import spawn_workers
from mvp_engine.utils.tracing import ProfilerConfig, StepTracer, TraceConfig

ROOT = Path(__file__).resolve().parent.parent


def test_disabled_tracer_hands_back_one_null_context(monkeypatch):
    monkeypatch.delenv("MVP_NVTX", raising=False)
    t = StepTracer.disabled()
    assert not t.enabled
    assert t.range("forward") is t.range("backward")
    t.begin_step(0)
    t.end_step(0)
    t.close()


def test_env_switch_turns_nvtx_on(monkeypatch):
    monkeypatch.setenv("MVP_NVTX", "1")
    t = StepTracer(TraceConfig())
    assert t.enabled and t.nvtx
    t.begin_step(3)
    with t.range("forward"):
        pass
    t.end_step(3)
    t.close()


class _FooBlock(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(4, 4)

    def forward(self, x):
        return self.lin(x)


def test_block_hooks_attach_to_blocks_only_and_detach():
    model = torch.nn.Sequential(_FooBlock(), torch.nn.ReLU(), _FooBlock())
    off = StepTracer(TraceConfig(nvtx=True))
    assert off.attach_blocks(model) == 0  # nvtx_blocks not asked for
    t = StepTracer(TraceConfig(nvtx=True, nvtx_blocks=True))
    assert t.attach_blocks(model) == 2
    ref = model(torch.ones(2, 4))
    t.close()
    assert all(not m._forward_hooks and not m._forward_pre_hooks for m in model.modules())
    named = StepTracer(TraceConfig(nvtx=True, nvtx_blocks=True, block_classes=["ReLU"]))
    assert named.attach_blocks(model) == 1
    assert torch.equal(model(torch.ones(2, 4)), ref)
    named.close()


def _profiled_run(rank, world, port, out_dir, shard=1):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import load_smoke_test_config

    root = ROOT / "recipes" / "qwen3"
    import_recipe_modules(root)
    over = ("model.pretrained_model_name_or_path=mvp/qwen3-tiny", "model.config_overrides.vocab_size=512",
            "model.config_overrides.num_hidden_layers=2", "optim.mixed_precision=fp32", "log.backends=[terminal]",
            "data.train_path=synthetic://text?vocab=512&min_len=16&max_len=96", "data.max_seq_len=128",
            "optim.global_batch_size=2", "model.gradient_checkpointing.enabled=false",
            "parallel.mesh.replicate=1", f"parallel.mesh.shard={shard}", "loop.total_steps=3", "dev_mode=true",
            "trace.profiler.enabled=true", "trace.profiler.wait=0", "trace.profiler.warmup=1",
            "trace.profiler.active=1", "trace.nvtx=true", "trace.nvtx_blocks=true")
    cfg = load_smoke_test_config(root, "synthetic_8b", output_dir=Path(out_dir), run_id="tr", config_overrides=over)
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    eng.train()
    return [str(p) for p in eng.tracer.traces]


def test_profiler_window_writes_a_trace_with_phase_labels(tmp_path):
    traces = spawn_workers(_profiled_run, 1, str(tmp_path), timeout=300)[0]
    assert len(traces) == 1 and Path(traces[0]).name == "rank0_step2.json"
    events = json.loads(Path(traces[0]).read_text())["traceEvents"]
    names = {e.get("name") for e in events}
    assert {"data", "forward", "backward", "optimizer"} <= names, sorted(n for n in names if n)[:40]


def test_each_rank_writes_its_own_trace(tmp_path):
    per_rank = spawn_workers(_profiled_run, 2, str(tmp_path), 2, timeout=300)
    assert [[Path(p).name for p in t] for t in per_rank] == [["rank0_step2.json"], ["rank1_step2.json"]]
    assert per_rank[0][0] != per_rank[1][0]


def test_profiler_config_bounds():
    import pytest
    from pydantic import ValidationError

    with pytest.raises(ValidationError):
        ProfilerConfig(active=0)
