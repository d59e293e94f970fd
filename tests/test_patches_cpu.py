"""Runtime patches: the registry's contract, and the FSDP2 recompute-cast patch against the torch this
engine runs on (gloo, CPU)."""

from __future__ import annotations

import enum
import types

import pytest
import torch

from mvp_engine.patches import PatchResult, apply_fsdp2_checkpoint_recompute_cast_patch


def _fsdp2_checkpoint_worker(rank, world, port, patch):
    """An FSDP2 submodule with a bf16 mixed-precision policy, run under non-reentrant checkpointing and
    fed fp32 inputs: the recompute in backward goes through FSDPState._pre_forward's early return."""
    import torch.nn as nn
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
    from torch.utils.checkpoint import checkpoint

    from mvp_engine.distributed.init import initialize_process_group

    initialize_process_group()
    result = apply_fsdp2_checkpoint_recompute_cast_patch() if patch else None
    mesh = init_device_mesh("cpu", (world,))

    class Root(nn.Module):
        def __init__(self):
            super().__init__()
            self.inner = nn.Linear(8, 8)
            self.head = nn.Linear(8, 1)

        def forward(self, x):
            return self.head(checkpoint(self.inner, x, use_reentrant=False).float())

    torch.manual_seed(0)
    m = Root()
    fully_shard(m.inner, mesh=mesh, mp_policy=MixedPrecisionPolicy(param_dtype=torch.bfloat16))
    fully_shard(m, mesh=mesh)  # root in fp32: only the checkpointed submodule computes in bf16
    try:
        m(torch.randn(4, 8)).sum().backward()
        outcome = "ok"
    except RuntimeError as exc:
        outcome = f"error: {exc}"
    grads = [getattr(p.grad, "full_tensor", lambda g=p.grad: g)() for p in m.parameters() if p.grad is not None]
    grads_finite = bool(grads) and all(bool(torch.isfinite(g).all()) for g in grads)
    return outcome, grads_finite, result


def test_fsdp2_recompute_under_checkpoint_needs_and_gets_the_cast():
    from mvp_engine.testing.utils import spawn_workers

    unpatched, _, _ = spawn_workers(_fsdp2_checkpoint_worker, 1, False, timeout=300)[0]
    # torch 2.11 skips the input cast on this path, so the recompute sees fp32 where the forward saw bf16;
    # a later torch may cast there (then there is nothing to fix)
    assert unpatched == "ok" or "metadata" in unpatched, unpatched
    patched, finite, result = spawn_workers(_fsdp2_checkpoint_worker, 1, True, timeout=300)[0]
    assert result.status == "applied" and patched == "ok" and finite, (patched, result)


class _State(enum.Enum):
    FORWARD = 1
    PRE_BACKWARD = 2


def _fake_state_module():
    class FSDPState:
        def __init__(self, state, cast=True):
            self._training_state = state
            self._mp_policy = types.SimpleNamespace(param_dtype=torch.bfloat16, cast_forward_inputs=cast)

        def _pre_forward(self, module, args, kwargs):
            return args, kwargs  # the legacy early return, for every state

    return types.SimpleNamespace(FSDPState=FSDPState, TrainingState=_State)


def test_patch_casts_only_on_the_recompute_path_and_is_idempotent():
    mod = _fake_state_module()
    assert apply_fsdp2_checkpoint_recompute_cast_patch(mod).status == "applied"
    assert apply_fsdp2_checkpoint_recompute_cast_patch(mod).status == "skipped"
    x, i = torch.randn(2), torch.arange(3)
    args, kwargs = mod.FSDPState(_State.PRE_BACKWARD)._pre_forward(None, (x, i), {"y": x})
    assert args[0].dtype == torch.bfloat16 and args[1].dtype == torch.long and kwargs["y"].dtype == torch.bfloat16
    args, _ = mod.FSDPState(_State.FORWARD)._pre_forward(None, (x,), {})
    assert args[0].dtype == torch.float32  # the normal forward path is left to torch
    args, _ = mod.FSDPState(_State.PRE_BACKWARD, cast=False)._pre_forward(None, (x,), {})
    assert args[0].dtype == torch.float32  # policy without input casting


def test_patch_skips_unknown_shapes():
    assert apply_fsdp2_checkpoint_recompute_cast_patch(types.SimpleNamespace()).status == "skipped"


def test_registry_disable_and_strict(monkeypatch):
    from mvp_engine.patches import registry

    monkeypatch.setenv("MVP_ENGINE_DISABLE_RUNTIME_PATCHES", "1")
    [r] = registry.apply_all_patches()
    assert r.status == "skipped" and "disabled" in r.reason
    monkeypatch.delenv("MVP_ENGINE_DISABLE_RUNTIME_PATCHES")

    def broken():
        raise ValueError("boom")

    monkeypatch.setattr(registry, "_PATCHES", [("broken", broken)])
    monkeypatch.setattr(registry, "_RESULTS", {})
    with pytest.warns(RuntimeWarning):
        [r] = registry.apply_all_patches()
    assert r == PatchResult("broken", "failed", "boom") and not r.applied
    monkeypatch.setattr(registry, "_RESULTS", {})
    monkeypatch.setenv("MVP_ENGINE_STRICT_RUNTIME_PATCHES", "1")
    with pytest.raises(RuntimeError, match="boom"):
        registry.apply_all_patches()
