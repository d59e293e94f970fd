"""Global-norm gradient clipping against torch's single-process clip: plain tensors, and DTensor gradients
of a torch FSDP2 model sharded over gloo ranks (the reference's backend path)."""

from __future__ import annotations

import torch

from mvp_engine.utils.training import clip_grad_norm_


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.GELU(), torch.nn.Linear(32, 8))


def _data():
    g = torch.Generator().manual_seed(1)
    return torch.randn(8, 16, generator=g), torch.randn(8, 8, generator=g)


def _reference(max_norm):
    m = _model()
    x, y = _data()
    torch.nn.functional.mse_loss(m(x), y).backward()
    norm = torch.nn.utils.clip_grad_norm_(m.parameters(), max_norm)
    return float(norm), [p.grad.clone() for p in m.parameters()]


def test_plain_parameters_match_torch():
    for max_norm in (1e-3, 1e6):  # clipped, and untouched
        norm_ref, grads_ref = _reference(max_norm)
        m = _model()
        x, y = _data()
        torch.nn.functional.mse_loss(m(x), y).backward()
        norm = clip_grad_norm_(m, max_norm)
        assert abs(float(norm) - norm_ref) <= 1e-6 * norm_ref
        for p, g in zip(m.parameters(), grads_ref):
            torch.testing.assert_close(p.grad, g)


def _fsdp2_worker(rank, world, port, max_norm):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.fsdp import fully_shard

    from mvp_engine.distributed.init import initialize_process_group

    initialize_process_group()
    mesh = init_device_mesh("cpu", (world,))
    m = _model()
    for layer in m:
        if isinstance(layer, torch.nn.Linear):
            fully_shard(layer, mesh=mesh)
    fully_shard(m, mesh=mesh)
    x, y = _data()
    # every rank sees the whole batch: FSDP averages identical gradients, so the result is the
    # single-process gradient
    torch.nn.functional.mse_loss(m(x), y).backward()
    norm = clip_grad_norm_(m, max_norm)
    return float(norm), [p.grad.full_tensor().clone() for p in m.parameters()]


def test_fsdp2_dtensor_gradients_match_single_process():
    from mvp_engine.testing.utils import spawn_workers

    norm_ref, grads_ref = _reference(1e-3)
    for norm, grads in spawn_workers(_fsdp2_worker, 2, 1e-3, timeout=300):
        assert abs(norm - norm_ref) <= 1e-5 * norm_ref
        for g, r in zip(grads, grads_ref):
            torch.testing.assert_close(g, r, rtol=1e-5, atol=1e-8)
