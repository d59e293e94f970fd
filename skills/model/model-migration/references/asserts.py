"""Skill asserts: a model family brought to this engine.

Copy to ``recipes/<recipe>/tests/skills/model-migration/asserts.py``.  A family plugs into the runtime
through a small contract rather than through HF classes: HF parameter names (checkpoints and
``hf_model/`` exports load unchanged), a meta-device build whose parameters the data-parallel runtime
materialises one at a time (``init_param_``), the recomputation switch, and the model's own FLOPs
formula, which the MFU log divides by.
"""

import torch

from mvp_engine.testing.skill_checks import expect_calls

_CONTRACT = ("calculate_model_flops", "gradient_checkpointing_enable", "init_param_")


def check_model_contract(model, *, seq_len=128):
    """Call from a model test on a (small) built model."""
    for name in _CONTRACT:
        assert callable(getattr(model, name, None)), f"{type(model).__name__} must implement {name}"
    names = [n for n, _ in model.named_parameters()]
    assert names and all(n.startswith(("model.", "lm_head.")) for n in names), (
        "parameter names must follow the HF layout (model.* and lm_head.*)")
    flops = float(model.calculate_model_flops(batch_size=1, seq_len=seq_len))
    # every weight outside the embedding table multiplies each token once in the forward (2 FLOPs per
    # weight and token); a training step's count (forward + backward) is at least that
    dense = sum(p.numel() for n, p in model.named_parameters() if "embed_tokens" not in n and p.dim() > 1)
    assert flops >= 2 * dense * seq_len, f"FLOPs formula too small: {flops:.3e} for {dense} matmul weights"


def test_engine_structure(engine_class):
    expect_calls(engine_class, "prepare_model", ["model_kit.build_model(", "apply_model_patches(", "random_init_seed"])


def assert_before_train_end(engine):
    model = engine.unwrapped_model
    for name in _CONTRACT:
        assert callable(getattr(model, name, None)), f"{type(model).__name__} must implement {name}"
    assert not any(p.is_meta for p in model.parameters() if isinstance(p, torch.Tensor) and p.numel()), (
        "every parameter must be materialised before training")
