"""Context parallelism on gloo ranks (CPU): ring and Ulysses attention, and a CP=2 model step,
against single-process attention / training on the whole sequence."""

import pytest
import torch

from mvp_engine.testing import spawn_workers


def _data(T, Hq, Hkv, D, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(T, Hq, D, generator=g)
    k = torch.randn(T, Hkv, D, generator=g)
    v = torch.randn(T, Hkv, D, generator=g)
    do = torch.randn(T, Hq, D, generator=g)
    # documents crossing chunk boundaries, a short one, and one spanning several chunks
    lens, left = [], T
    for n in (5, 23, 1, 40, 9):
        if left <= 0:
            break
        lens.append(min(n, left))
        left -= lens[-1]
    if left > 0:
        lens.append(left)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    return q, k, v, do, cu


def _cp_attention(rank, world, port, impl, T, Hq, Hkv):
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import PackedContext
    from mvp_engine.parallel.context import ContextParallel

    initialize_process_group()
    q, k, v, do, cu = _data(T, Hq, Hkv, 16, 0)
    cp = ContextParallel(dist.group.WORLD, impl=impl)
    idx = cp.local_indices(T)
    ql, kl, vl = (t[idx].clone().requires_grad_() for t in (q, k, v))
    ctx = PackedContext(torch.zeros(1, len(idx), dtype=torch.long), cu, int((cu[1:] - cu[:-1]).max()), None, cp=cp)
    o = cp.attention(ql, kl, vl, ctx, 16**-0.5)
    o.backward(do[idx])
    return idx, o.detach(), ql.grad, kl.grad, vl.grad


@pytest.mark.parametrize("impl,world", [("ring", 2), ("ring", 4), ("ulysses", 2), ("ulysses", 4)])
def test_context_parallel_attention_matches_full(impl, world):
    from mvp_engine.ops.attention import attention_reference

    T, Hq, Hkv = 96, 8, 4
    q, k, v, do, cu = _data(T, Hq, Hkv, 16, 0)
    qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
    ref = attention_reference(qq, kk, vv, cu, causal=True, softmax_scale=16**-0.5)
    ref.backward(do)
    out = spawn_workers(_cp_attention, world, impl, T, Hq, Hkv, timeout=300)
    o = torch.zeros_like(q)
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    for idx, ol, gq, gk, gv in out:
        o[idx], dq[idx], dk[idx], dv[idx] = ol, gq, gk, gv
    torch.testing.assert_close(o, ref.detach(), atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(dq, qq.grad, atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(dk, kk.grad, atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(dv, vv.grad, atol=2e-5, rtol=1e-4)


def _cp_model_step(rank, world, port, impl, reshard=False):
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.kit.llm.data.collator import varlen_metadata
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.parallel.context import ContextParallel
    from mvp_engine.parallel.fsdp import NativeFSDP

    if world > 1:
        initialize_process_group()
    model = build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=256, hidden_size=64, intermediate_size=128,
                        num_attention_heads=4, num_key_value_heads=2, num_hidden_layers=2)
    g = torch.Generator().manual_seed(11)
    T = 64
    ids = torch.randint(0, 256, (1, T), generator=g)
    seg = torch.tensor([[1] * 20 + [2] * 30 + [3] * 14])
    cu, mx, pos = varlen_metadata(seg)
    batch = {"input_ids": ids, "labels": ids.clone(), "pack_segment_ids": seg, "cu_seq_lens_q": cu,
             "max_length_q": mx, "position_ids": pos}
    group = dist.group.WORLD if world > 1 else None
    if world > 1:
        model._mvp_cp = ContextParallel(group, impl=impl)
        batch = model._mvp_cp.shard_batch(batch)
    fsdp = NativeFSDP(model, group=group, device=torch.device("cpu"), param_dtype=torch.float32,
                      reshard_after_forward=reshard and world > 1)
    assert sum(u.resharded for u in fsdp.units) == (2 if reshard and world > 1 else 0)
    keys = ("input_ids", "labels", "shift_labels", "position_ids", "cu_seq_lens_q", "max_length_q")
    out = fsdp(**{k: batch[k] for k in keys if k in batch})
    loss_sum = out["loss"].sum()
    loss_sum.backward()
    fsdp.finish_grad_sync()
    total = loss_sum.detach().clone()
    if world > 1:
        dist.all_reduce(total)
    sd = fsdp.checkpoint_state_dict(full=True)  # parameters only; grads checked via the shard norm below
    gn = fsdp.clip_grad_norm_(1e9)
    return float(total), float(gn)


@pytest.mark.parametrize("reshard", [False, True])
@pytest.mark.parametrize("impl", ["ring", "ulysses"])
def test_context_parallel_model_step_matches_single_process(impl, reshard):
    """Context-parallel ranks (sharing the parameters, resident or resharded after each use) reproduce the
    single-process loss and gradient norm."""
    single = spawn_workers(_cp_model_step, 1, impl, timeout=300)[0]
    multi = spawn_workers(_cp_model_step, 2, impl, reshard, timeout=300)
    for loss, gn in multi:
        assert abs(loss - single[0]) < 1e-4 * abs(single[0]), (loss, single)
        # gradients are averaged over the 2 ranks: the norm of the mean is half the summed norm
        assert abs(2 * gn - single[1]) < 2e-4 * single[1], (gn, single)


def _cp_tp_step(rank, world, port, impl, tp, cp, sp):
    """One forward + backward of a tiny Qwen3 through the public wrapping (mesh -> parallelize_model ->
    host-side batch cut), on a context x tensor mesh."""
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.distributed.parallel_mesh import ParallelMesh
    from mvp_engine.distributed.parallelize import parallelize_model
    from mvp_engine.kit.llm.data.collator import varlen_metadata
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.parallel.context import maybe_shard_batch

    if world > 1:
        initialize_process_group()
    mesh = ParallelMesh.initialize("cpu", {"replicate": 1, "shard": 1, "context": cp, "tensor": tp})
    model = build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=256, hidden_size=64, intermediate_size=128,
                        num_attention_heads=8, num_key_value_heads=4, num_hidden_layers=2, head_dim=16)
    g = torch.Generator().manual_seed(11)
    T = 64
    ids = torch.randint(0, 256, (1, T), generator=g)
    seg = torch.tensor([[1] * 20 + [2] * 30 + [3] * 14])
    cu, mx, pos = varlen_metadata(seg)
    batch = {"input_ids": ids, "labels": ids.clone(), "pack_segment_ids": seg, "cu_seq_lens_q": cu,
             "max_length_q": mx, "position_ids": pos}
    wrapped = parallelize_model(model, parallel_mesh=mesh, device=torch.device("cpu"),
                                backend_kwargs={"impl": "native", "sequence_parallel": sp,
                                                "context_parallel": {"impl": impl}, "comm": {"fused": False}})
    batch = maybe_shard_batch(model, batch)
    keys = ("input_ids", "labels", "shift_labels", "position_ids", "cu_seq_lens_q", "max_length_q")
    loss = wrapped(**{k: batch[k] for k in keys if k in batch})["loss"].sum()
    loss.backward()
    total = loss.detach().clone()
    if world > 1:
        dist.all_reduce(total, group=mesh.dp_cp.group)  # context ranks hold different tokens
        if sp:
            dist.all_reduce(total, group=mesh.tp.group)  # and so do sequence-parallel tensor ranks
    return float(total), float(wrapped.clip_grad_norm_(1e9))


@pytest.mark.parametrize("sp", [False, True])
@pytest.mark.parametrize("impl", ["ring", "ulysses"])
def test_context_parallel_composes_with_tensor_parallel(impl, sp):
    """context 2 x tensor 2 (with and without sequence parallelism) against one process: the same loss, and
    the gradient norm of the average over the two context ranks (half the one-process norm)."""
    single = spawn_workers(_cp_tp_step, 1, impl, 1, 1, False, timeout=300)[0]
    for loss, gn in spawn_workers(_cp_tp_step, 4, impl, 2, 2, sp, timeout=300):
        assert abs(loss - single[0]) < 1e-4 * abs(single[0]), (loss, single)
        assert abs(2 * gn - single[1]) < 2e-4 * single[1], (gn, single)
