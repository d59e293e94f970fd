"""Skill asserts: packing multimodal samples.

Copy to ``recipes/<recipe>/tests/skills/vlm-packing/asserts.py``.  Samples are packed whole (a sample and
its images are never split across packs) into ``data.max_seq_len`` tokens; every packed document is its
own attention block (``block_causal``), which the engine expresses as varlen ``cu_seq_lens_q`` rather
than a dense mask.
"""

import torch

from mvp_engine.testing.skill_checks import config_get, phase_source


def test_config_structure(config):
    assert int(config_get(config, "data.max_seq_len", 0)) > 0
    strategy = config_get(config, "data.packing_selection_strategy", "best_fit")
    assert strategy in ("random", "best_fit"), strategy
    assert int(config_get(config, "data.packing_open_pack_limit", 1)) >= 1
    assert int(config_get(config, "data.packing_buffer_size", 0)) >= 0


def test_engine_structure(engine_class):
    src = phase_source(engine_class, "_data_spec") or phase_source(engine_class, "prepare_dataloader")
    for needle in ("MLLMPackingSpec(", "max_seq_len=", "selection_strategy=", "open_pack_limit=", "buffer_size=",
                   "block_causal=True"):
        assert needle in src, f"the packing spec must set {needle}"


def assert_train_pre_step_end(engine, ctx):
    data = ctx.data
    ids = data["input_ids"]
    limit = int(config_get(engine.config, "data.max_seq_len"))
    assert ids.shape[-1] <= limit, f"pack of {ids.shape[-1]} tokens exceeds max_seq_len {limit}"
    cu = torch.as_tensor(data["cu_seq_lens_q"]).cpu()
    assert int(cu[0]) == 0 and int(cu[-1]) == ids.numel(), "document boundaries must cover the packed rows"
    assert bool((cu[1:] >= cu[:-1]).all()), "document boundaries must be non-decreasing"
    assert int(data["max_length_q"]) == int((cu[1:] - cu[:-1]).max()), "max_length_q is the longest document"
