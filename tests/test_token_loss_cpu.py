"""TokenNormedLossKit: the accumulated, rescaled gradient is the gradient of the step's mean token loss,
independent of how the tokens are split into micro-batches and ranks; the spike guard decides alike on
every rank."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from mvp_engine.kit.loss.token_loss import TokenNormedLossKit


def _batches(seed: int, n: int, vocab: int = 11, dim: int = 6):
    g = torch.Generator().manual_seed(seed)
    out = []
    for k in range(n):
        T = 5 + 3 * k
        x = torch.randn(T, dim, generator=g)
        y = torch.randint(0, vocab, (T,), generator=g)
        y[torch.rand(T, generator=g) < 0.3] = -100  # unsupervised positions
        out.append((x, y))
    return out


def _model(vocab: int = 11, dim: int = 6) -> torch.nn.Linear:
    torch.manual_seed(0)
    return torch.nn.Linear(dim, vocab)


def _token_losses(model, x, y):
    return F.cross_entropy(model(x), y, ignore_index=-100, reduction="none")


def _kit_grads(model, batches, divisor, *, group=None, world=1):
    kit = TokenNormedLossKit(device=torch.device("cpu"), dp_world_size=world, dp_group=group)
    for x, y in batches:
        per_tok = _token_losses(model, x, y)
        eff = int((y != -100).sum())
        loss = kit.accumulate_microbatch(loss_sum=per_tok.sum(), effective_tokens=eff, total_tokens=len(y),
                                         backward_divisor=divisor)
        loss.backward()
    stats = kit.reduce_window()
    kit.rescale_gradients(model.parameters(), stats)
    return stats


def _reference_grads(model, batches):
    xs = torch.cat([x for x, _ in batches])
    ys = torch.cat([y for _, y in batches])
    F.cross_entropy(model(xs), ys, ignore_index=-100, reduction="mean").backward()
    return [p.grad.clone() for p in model.parameters()]


def test_micro_batch_split_does_not_change_the_gradient():
    batches = _batches(1, 4)
    ref_model = _model()
    ref = _reference_grads(ref_model, batches)
    for split, divisor in (([batches], 64), ([batches[:2], batches[2:]], 40), ([[b] for b in batches], 17)):
        model = _model()
        flat = [b for part in split for b in part]
        stats = _kit_grads(model, flat, divisor)
        assert stats.global_effective_tokens == sum(int((y != -100).sum()) for _, y in batches)
        assert stats.global_total_tokens == sum(len(y) for _, y in batches)
        for p, r in zip(model.parameters(), ref):
            torch.testing.assert_close(p.grad, r, rtol=1e-5, atol=1e-7)
        mean = stats.global_loss_sum / stats.global_effective_tokens
        with torch.no_grad():
            xs = torch.cat([x for x, _ in batches])
            ys = torch.cat([y for _, y in batches])
            want = float(F.cross_entropy(ref_model(xs), ys, ignore_index=-100))
        assert abs(mean - want) < 1e-5


def _dp_worker(rank, world, port, spike_rank):
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group

    initialize_process_group()
    batches = _batches(10 + rank, 2 + rank)  # ranks hold different numbers of micro-batches' tokens
    model = _model()
    _kit_grads(model, batches, divisor=32, group=dist.group.WORLD, world=world)
    for p in model.parameters():  # what data parallelism does: average the gradients over ranks
        dist.all_reduce(p.grad)
        p.grad /= world
    grads = [p.grad.clone() for p in model.parameters()]

    # the guard: rank `spike_rank` feeds a huge loss; every rank must take the same decision
    kit = TokenNormedLossKit(device=torch.device("cpu"), dp_world_size=world, dp_group=dist.group.WORLD)
    kit.build_loss_guard(spike_multiplier=3.0, window_size=4, min_history=2)
    decisions = []
    for step, base in enumerate([1.0, 1.1, 0.9, 1.0]):
        val = 1000.0 if (step == 3 and rank == spike_rank) else base
        decisions.append(kit.guard_loss(torch.tensor(val * 10), 10, step=step))
    return grads, decisions


def test_data_parallel_gradient_is_the_global_token_mean():
    from mvp_engine.testing.utils import spawn_workers

    out = spawn_workers(_dp_worker, 2, 0, timeout=300)
    everything = _batches(10, 2) + _batches(11, 3)
    ref = _reference_grads(_model(), everything)
    for grads, decisions in out:
        for g, r in zip(grads, ref):
            torch.testing.assert_close(g, r, rtol=1e-5, atol=1e-7)
        # steps 0-1 fill the history, step 2 passes, step 3 is a spike on rank 0 only: both ranks skip it
        assert decisions == [True, True, True, False]
