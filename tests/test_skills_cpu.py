"""The skills' assert templates and run summariser, checked against this repository's recipes.

Each ``skills/**/references/asserts.py`` is meant to be copied into a recipe's ``tests/skills/<id>/``;
here every template is run against the recipe engines it describes (structure checks), against engines
that break its rule (it must fail), and around real CPU training runs (runtime hooks).
"""

from __future__ import annotations

import importlib.util
import json
import subprocess
import sys
from pathlib import Path

import pytest
import yaml

ROOT = Path(__file__).resolve().parent.parent
SKILLS = ROOT / "skills"


def _template(skill: str):
    path = SKILLS / skill / "references" / "asserts.py"
    spec = importlib.util.spec_from_file_location(f"skill_{skill.replace('/', '_').replace('-', '_')}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _engine(recipe: str, name: str):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules

    import_recipe_modules(ROOT / "recipes" / recipe)
    return ENGINE_REGISTRY.get(name)


def _configs(recipe: str, engine_cls):
    """Every config of the recipe as the engine sees it: merged over the defaults, validated, dumped."""
    from mvp_engine.config.loader import deep_merge, load_yaml

    default = load_yaml(ROOT / "mvp_engine" / "config" / "default.yaml")
    paths = sorted((ROOT / "recipes" / recipe / "configs").glob("*.yaml"))
    return [engine_cls.ConfigClass.model_validate(deep_merge(default, yaml.safe_load(p.read_text()))).model_dump()
            for p in paths]


TEXT = ["training/token-normalized-loss", "training/loss-spike-guard", "training/model-flops-utilization",
        "training/failure-recovery", "model/gradient-checkpointing", "model/model-compile", "model/model-migration",
        "model/liger-kernel", "parallel/tensor-parallel", "parallel/sequence-parallel", "parallel/native-fsdp",
        "parallel/context-parallel", "parallel/fsdp2-prefetching", "recipe/new-recipe-template"]
VISION = ["training/token-normalized-loss", "training/loss-spike-guard", "training/model-flops-utilization",
          "training/failure-recovery", "model/gradient-checkpointing", "model/model-compile", "model/model-migration",
          "model/vlm-freeze-policy", "parallel/native-fsdp", "data/vlm-data-pipeline", "data/vlm-packing",
          "recipe/new-recipe-template"]
CASES = [("qwen3", "Qwen3Engine", s) for s in TEXT] + [("qwen3_vl", "Qwen3VLEngine", s) for s in VISION] + \
        [("openbee", "OpenBeeEngine", s) for s in VISION]


def test_every_template_is_listed():
    found = {str(p.parent.parent.relative_to(SKILLS)) for p in SKILLS.glob("**/references/asserts.py")}
    assert found == set(TEXT) | set(VISION), found ^ (set(TEXT) | set(VISION))


@pytest.mark.parametrize("recipe,engine,skill", CASES)
def test_template_accepts_recipe(recipe, engine, skill):
    mod = _template(skill)
    cls = _engine(recipe, engine)
    if hasattr(mod, "test_file_structure"):
        mod.test_file_structure(ROOT / "recipes" / recipe)
    if hasattr(mod, "test_engine_structure"):
        mod.test_engine_structure(cls)
    if hasattr(mod, "test_config_structure"):
        for cfg in _configs(recipe, cls):
            mod.test_config_structure(cfg)


# ------------------------------------------------------------------ templates reject broken engines
def _broken_engines():
    Qwen3Engine = _engine("qwen3", "Qwen3Engine")

    class ClipBeforeRescale(Qwen3Engine):  # clips the unscaled-by-tokens gradient
        def optimizer_step(self, ctx):
            stats = self.token_loss_kit.reduce_window()
            self.scaler.unscale_(self.optimizer)
            clip_grad_norm_(self.model, 1.0)  # noqa: F821 - never executed
            self.token_loss_kit.rescale_gradients(self.model, stats)
            self.scaler.step(self.optimizer)
            self.token_loss_kit.reset()

    class SkipsBackward(Qwen3Engine):  # a skipped micro-batch leaves early: the collectives would hang
        def backward_step(self, ctx):
            loss_sum = ctx.outputs["loss"].sum()
            if not self.token_loss_kit.guard_loss(loss_sum, 1, step=0):
                loss_sum = loss_sum * 0.0
                return
            ctx.loss = self.token_loss_kit.accumulate_microbatch(loss_sum=loss_sum, effective_tokens=1,
                                                                 total_tokens=1, backward_divisor=1)
            ctx.loss.backward()

    class CheckpointAfterWrap(Qwen3Engine):  # recomputation switched on after the runtime built its units
        def prepare_model(self):
            m = self.config.model
            model = self.model_kit.build_model(m.pretrained_model_name_or_path, random_init_seed=0)
            model = self.model_kit.apply_model_patches(model, [])
            model = self.model_kit.apply_freeze_policy(model)
            model = parallelize_model(model, parallel_mesh=self.parallel_mesh,  # noqa: F821
                                      backend_kwargs={})
            if m.gradient_checkpointing.enabled:
                self.model_kit.apply_gradient_checkpointing(model, use_reentrant=m.gradient_checkpointing.use_reentrant,
                                                            num_layers=m.gradient_checkpointing.num_layers)
            return model

    class NoMFU(Qwen3Engine):
        def forward_step(self, ctx):
            ctx.outputs = {"loss": self.model(**ctx.data)["loss"], "logs": {}}

    return {"training/token-normalized-loss": ClipBeforeRescale, "training/loss-spike-guard": SkipsBackward,
            "model/gradient-checkpointing": CheckpointAfterWrap, "training/model-flops-utilization": NoMFU}


@pytest.mark.parametrize("skill", ["training/token-normalized-loss", "training/loss-spike-guard",
                                   "model/gradient-checkpointing", "training/model-flops-utilization"])
def test_template_rejects_broken_engine(skill):
    with pytest.raises(AssertionError):
        _template(skill).test_engine_structure(_broken_engines()[skill])


def test_config_templates_reject_bad_configs():
    with pytest.raises(AssertionError):
        _template("parallel/sequence-parallel").test_config_structure(
            {"parallel": {"mesh": {"tensor": 1}, "backend_kwargs": {"sequence_parallel": True}}})
    with pytest.raises(AssertionError):
        _template("parallel/context-parallel").test_config_structure(
            {"parallel": {"mesh": {"context": 4}, "backend_kwargs": {"context_parallel": {"impl": "ring"}}},
             "data": {"max_seq_len": 1020}})
    with pytest.raises(AssertionError):
        _template("model/vlm-freeze-policy").test_config_structure(
            {"model": {"freeze_vit": True, "freeze_projector": True, "freeze_llm": True}})


def test_model_migration_contract_on_tiny_qwen3():
    from mvp_engine.models.qwen3 import build_qwen3

    model = build_qwen3("mvp/qwen3-tiny", seed=0, vocab_size=512, num_hidden_layers=2)
    _template("model/model-migration").check_model_contract(model, seq_len=64)


def test_liger_report_check():
    from mvp_engine.kit.model.liger import LigerKernelKit, LigerPatch

    mod = _template("model/liger-kernel")
    patches = {"rms_norm": LigerPatch("json", "dumps", json.dumps),  # rebinding to itself: harmless
               "cross_entropy": LigerPatch("json", "loads", None)}      # excluded by default: not applied
    report = LigerKernelKit().apply(model_family="custom", custom_patches=patches)
    assert report.route == "custom" and report.patched == ("json.dumps",) and json.loads("1") == 1
    mod.check_report(report)
    assert LigerKernelKit().apply(model_family="qwen3").route == "official"
    with pytest.raises(ValueError, match="custom_patches"):
        LigerKernelKit().apply(model_family="llama")


# ------------------------------------------------------------------ runtime hooks on real CPU runs
TEXT_RUNTIME = ["training/token-normalized-loss", "training/loss-spike-guard", "training/model-flops-utilization",
                "training/failure-recovery", "model/gradient-checkpointing", "model/model-migration",
                "parallel/tensor-parallel", "parallel/sequence-parallel", "parallel/native-fsdp",
                "parallel/context-parallel", "parallel/fsdp2-prefetching"]
VISION_RUNTIME = ["training/token-normalized-loss", "model/vlm-freeze-policy", "data/vlm-data-pipeline",
                  "data/vlm-packing", "parallel/native-fsdp"]


def _run_with_hooks(rank, world, port, recipe, config, overrides, skills, out_dir):
    from mvp_engine.engine import ENGINE_REGISTRY
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.testing.utils import inject_engine_assert_hooks, load_smoke_test_config

    root = ROOT / "recipes" / recipe
    import_recipe_modules(root)
    cfg = load_smoke_test_config(root, config, output_dir=Path(out_dir), run_id="skills",
                                 config_overrides=tuple(overrides))
    eng = ENGINE_REGISTRY.get(cfg["engine"])(cfg)
    calls = {"steps": 0}

    class _Counter:  # proves the hooks run: counts completed optimizer steps seen by a hook
        @staticmethod
        def assert_train_post_step_end(ctx):
            calls["steps"] += int(bool(ctx.optimizer_step_completed))

    inject_engine_assert_hooks(eng, [_template(s) for s in skills] + [_Counter])
    eng.train()
    return dict(eng.last_logs, hook_steps=calls["steps"])


_TINY_QWEN3 = ("model.pretrained_model_name_or_path=mvp/qwen3-tiny", "model.config_overrides.vocab_size=512",
               "model.config_overrides.num_hidden_layers=2", "optim.mixed_precision=fp32",
               "data.train_path=synthetic://text?vocab=512&min_len=16&max_len=96", "data.max_seq_len=128",
               "model.gradient_checkpointing.enabled=true", "model.gradient_checkpointing.num_layers=1")


def test_text_runtime_hooks_and_run_summary(tmp_path):
    from mvp_engine.testing.utils import spawn_workers

    over = _TINY_QWEN3 + ("loop.total_steps=3", "checkpoint.interval=2", "checkpoint.keep_n=1", "dev_mode=false",
                          "log.backends=[file]", "optim.global_batch_size=4", "optim.loss_spike_skip_multiplier=50.0")
    logs = spawn_workers(_run_with_hooks, 2, "qwen3", "synthetic_8b", over, TEXT_RUNTIME, str(tmp_path), timeout=900)
    assert logs[0]["tokens/effective"] > 0 and logs[0]["train/loss"] == pytest.approx(logs[1]["train/loss"])
    assert [lg["hook_steps"] for lg in logs] == [3, 3]

    run_dir = tmp_path / "skills"
    script = SKILLS / "experiment" / "experiment-analysis" / "scripts" / "summarize_run.py"
    out = subprocess.run([sys.executable, str(script), "--run-dir", str(run_dir), "--window", "2"],
                         capture_output=True, text=True, check=True).stdout
    summary = json.loads(out)
    assert summary["run"]["engine"] == "Qwen3Engine"
    assert summary["metrics"]["train/loss"]["count"] == 3
    assert summary["metrics"]["train/loss"]["last"]["step"] == 3
    assert summary["health"]["finished"] and not summary["health"]["non_finite"]
    ck = summary["checkpoints"]
    assert ck["latest_complete"] == "iter_3" and ck["incomplete"] == [], ck
    assert [c["name"] for c in ck["directories"]] == ["iter_3"], "keep_n=1 keeps only the newest checkpoint"


def test_vision_runtime_hooks(tmp_path):
    from mvp_engine.testing.utils import spawn_workers

    over = ("loop.total_steps=2", "checkpoint.interval=1000000", "optim.global_batch_size=2",
            "model.freeze_vit=true")
    logs = spawn_workers(_run_with_hooks, 1, "qwen3_vl", "synthetic_tiny", over, VISION_RUNTIME, str(tmp_path),
                         timeout=900)
    assert logs[0]["tokens/effective"] > 0 and logs[0]["hook_steps"] == 2
