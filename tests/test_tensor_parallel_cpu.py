"""Native tensor parallelism (with and without sequence parallelism) on gloo ranks vs one process."""

import pytest
import torch

from mvp_engine.testing import spawn_workers


def _train(rank, world, port, tp_size, sp, steps, dp_rows=None, reshard=False):
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.kit.llm.data.collator import varlen_metadata
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.optim import FlatAdamW
    from mvp_engine.parallel.tensor_parallel import apply_native_tensor_parallel

    if world > 1:
        initialize_process_group()
    model = build_qwen3("mvp/qwen3-tiny", seed=5, vocab_size=256, hidden_size=64, intermediate_size=128,
                        num_attention_heads=4, num_key_value_heads=2, num_hidden_layers=2)
    dp_group = tp_group = None
    if world > 1:
        ranks = list(range(world))
        tp_groups = [dist.new_group(ranks[i:i + tp_size]) for i in range(0, world, tp_size)]
        dp_groups = [dist.new_group(ranks[i::tp_size]) for i in range(tp_size)]
        tp_group = tp_groups[rank // tp_size]
        dp_group = dp_groups[rank % tp_size] if world // tp_size > 1 else None
        apply_native_tensor_parallel(model, group=tp_group, sequence_parallel=sp)
    dp = dp_rows or world // tp_size
    fsdp = NativeFSDP(model, group=dp_group, device=torch.device("cpu"), param_dtype=torch.float32,
                      tp_group=tp_group, reshard_after_forward=reshard)
    assert sum(u.resharded for u in fsdp.units) == (2 if reshard else 0)
    opt = FlatAdamW(fsdp, lr=1e-2, weight_decay=0.0)
    g = torch.Generator().manual_seed(9)
    T = 64
    seg = torch.tensor([[1] * 24 + [2] * 40])
    cu, mx, pos = varlen_metadata(seg)
    losses, norms = [], []
    for _ in range(steps):
        ids = torch.randint(0, 256, (dp, T), generator=g)
        row = ids[rank // tp_size:rank // tp_size + 1] if world > 1 else ids
        if world == 1 and dp == 1:
            row = ids
        total = 0.0
        rows = [row] if world > 1 else [ids[i:i + 1] for i in range(ids.shape[0])]
        for r_ in rows:
            out = fsdp(input_ids=r_, labels=r_, position_ids=pos, cu_seq_lens_q=cu, max_length_q=mx)
            l = out["loss"].sum() / ((T - 1) * (1 if world > 1 else len(rows)))
            l.backward()
            total += float(l.detach())
        s = torch.tensor([total])
        if world > 1:
            if sp:
                dist.all_reduce(s, group=tp_group)  # each tensor rank holds 1/tp of the tokens
            if dp_group is not None:
                dist.all_reduce(s, group=dp_group)
                s /= dp
        n = fsdp.clip_grad_norm_(1e9)
        opt.step()
        losses.append(float(s))
        norms.append(float(n))
    return losses, norms


@pytest.mark.parametrize("world,tp,sp,reshard", [(2, 2, True, False), (2, 2, False, False), (4, 2, True, False),
                                                (4, 2, True, True)])
def test_tensor_parallel_matches_single_process(world, tp, sp, reshard):
    """Tensor (+ sequence) parallel ranks, with data parallelism over the tensor groups when world > tp and
    optionally resharded weights, reproduce one process that sees the data-parallel rows as micro-batches
    of the same optimizer step: losses and gradient norms over three AdamW steps."""
    dp = world // tp
    single = spawn_workers(_train, 1, 1, False, 3, dp, timeout=300)[0]
    multi = spawn_workers(_train, world, tp, sp, 3, None, reshard, timeout=300)
    for losses, norms in multi:
        for a, b in zip(losses, single[0]):
            assert abs(a - b) < 2e-4 * abs(b), (losses, single[0])
        for a, b in zip(norms, single[1]):
            assert abs(a - b) < 2e-3 * abs(b), (norms, single[1])


def _hsdp_tp_step(rank, world, port, rep, shard, tp, sp, reshard):
    """One forward + backward through the public wrapping on a replicate x shard x tensor mesh; every
    data-parallel rank feeds the same row, so the averaged gradient is the one-process gradient."""
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.distributed.parallel_mesh import ParallelMesh
    from mvp_engine.distributed.parallelize import parallelize_model
    from mvp_engine.kit.llm.data.collator import varlen_metadata
    from mvp_engine.models.qwen3 import build_qwen3

    if world > 1:
        initialize_process_group()
    mesh = ParallelMesh.initialize("cpu", {"replicate": rep, "shard": shard, "context": 1, "tensor": tp})
    model = build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=256, hidden_size=64, intermediate_size=128,
                        num_attention_heads=8, num_key_value_heads=4, num_hidden_layers=2, head_dim=16)
    g = torch.Generator().manual_seed(11)
    T = 64
    ids = torch.randint(0, 256, (1, T), generator=g)
    seg = torch.tensor([[1] * 20 + [2] * 30 + [3] * 14])
    cu, mx, pos = varlen_metadata(seg)
    wrapped = parallelize_model(model, parallel_mesh=mesh, device=torch.device("cpu"),
                                backend_kwargs={"impl": "native", "sequence_parallel": sp, "comm": {"fused": False},
                                                "reshard_after_forward": reshard})
    loss = wrapped(input_ids=ids, labels=ids.clone(), position_ids=pos, cu_seq_lens_q=cu,
                   max_length_q=mx)["loss"].sum()
    loss.backward()
    total = loss.detach().clone()
    if sp:
        dist.all_reduce(total, group=mesh.tp.group)  # each tensor rank holds the losses of 1/tp of the tokens
    return float(total), float(wrapped.clip_grad_norm_(1e9)), wrapped.rep_world


@pytest.mark.parametrize("sp,reshard", [(False, False), (True, True)])
def test_hsdp_composes_with_tensor_parallel(sp, reshard):
    """replicate 2 x shard 2 x tensor 2 (8 gloo ranks): HSDP is active and loss and gradient norm equal
    the one-process run."""
    single = spawn_workers(_hsdp_tp_step, 1, 1, 1, 1, False, False, timeout=300)[0]
    for loss, gn, rep_world in spawn_workers(_hsdp_tp_step, 8, 2, 2, 2, sp, reshard, timeout=600):
        assert rep_world == 2
        assert abs(loss - single[0]) < 1e-4 * abs(single[0]) and abs(gn - single[1]) < 2e-4 * single[1]
