"""Native flat FSDP on gloo ranks (CPU): world 2 must reproduce the single-process run."""

import pytest
import torch

from mvp_engine.testing import spawn_workers


def _train(rank, world, port, steps, seed, tied=False):
    import os

    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.optim import FlatAdamW

    if world > 1:
        initialize_process_group()
    group = dist.group.WORLD if world > 1 else None
    model = build_qwen3("mvp/qwen3-tiny", seed=seed, vocab_size=256, hidden_size=128, intermediate_size=256,
                        num_attention_heads=2, num_key_value_heads=1, tie_word_embeddings=tied)
    if tied:
        assert model.lm_head.weight is model.model.embed_tokens.weight
    fsdp = NativeFSDP(model, group=group, device=torch.device("cpu"), param_dtype=torch.float32)
    opt = FlatAdamW(fsdp, lr=1e-3, weight_decay=0.1)
    g = torch.Generator().manual_seed(123)
    data = [torch.randint(0, 256, (2, 64), generator=g) for _ in range(steps)]
    losses = []
    for x in data:
        # each rank takes its half of the global batch of 2 rows
        rows = x if world == 1 else x[rank:rank + 1]
        out = fsdp(input_ids=rows, labels=rows)
        loss = out["loss"].sum() / (rows.shape[0] * (rows.shape[1] - 1))  # rank-local mean; ranks are averaged
        loss.backward()
        fsdp.clip_grad_norm_(1.0)
        opt.step()
        l = loss.detach().clone()
        if world > 1:
            dist.all_reduce(l)
            l /= world
        losses.append(float(l))
    sd = fsdp.checkpoint_state_dict(full=True)
    return losses, {k: v.clone() for k, v in list(sd.items())[:4]}


@pytest.mark.parametrize("tied", [False, True])
def test_fsdp_world2_matches_single_process(tied):
    """World 2 against one process over 5 AdamW steps with clipping; ``tied``: the LM head shares the
    embedding matrix (the small Qwen3 presets), one flat-buffer entry under two names."""
    single = spawn_workers(_train, 1, 5, 7, tied)[0]
    multi = spawn_workers(_train, 2, 5, 7, tied)
    for a, b in zip(single[0], multi[0][0]):
        assert abs(a - b) < 2e-3 * max(1.0, abs(a)), (single[0], multi[0][0])
    assert multi[0][0] == multi[1][0]
    for k, v in single[1].items():
        assert torch.allclose(v, multi[0][1][k], atol=1e-4), k
        assert torch.allclose(multi[0][1][k], multi[1][1][k])


def _train_reshard(rank, world, port, steps, reshard, ckpt):
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.optim import FlatAdamW

    initialize_process_group()
    model = build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=256, hidden_size=128, intermediate_size=256,
                        num_attention_heads=2, num_key_value_heads=1, num_hidden_layers=5)
    if ckpt:
        model.gradient_checkpointing_enable({"num_layers": 3})
    fsdp = NativeFSDP(model, group=dist.group.WORLD, device=torch.device("cpu"), param_dtype=torch.float32,
                      reshard_after_forward=reshard)
    assert sum(u.resharded for u in fsdp.units) == (5 if reshard else 0)
    opt = FlatAdamW(fsdp, lr=1e-3, weight_decay=0.1)
    g = torch.Generator().manual_seed(321)
    losses = []
    for _ in range(steps):
        total = 0.0
        for micro in range(2):  # two micro-batches per step: gradients accumulate across them
            x = torch.randint(0, 256, (2, 48), generator=g)[rank:rank + 1]
            fsdp.set_requires_gradient_sync(micro == 1)
            out = fsdp(input_ids=x, labels=x)
            loss = out["loss"].sum() / (2 * 47)
            loss.backward()
            total += float(loss.detach())
        fsdp.clip_grad_norm_(1.0)
        opt.step()
        losses.append(total)
    sd = fsdp.checkpoint_state_dict(full=True)
    return losses, {k: v.clone() for k, v in sd.items() if "layers.2" in k or "layers.4" in k}


def test_resharded_weights_match_resident_weights():
    """reshard_after_forward (full weights only while a block runs, gathered again for backward and for
    recomputation) reproduces the resident run, with accumulation and activation checkpointing."""
    for ckpt in (False, True):
        resident = spawn_workers(_train_reshard, 2, 4, False, ckpt)
        resharded = spawn_workers(_train_reshard, 2, 4, True, ckpt)
        for r in range(2):
            for a, b in zip(resident[r][0], resharded[r][0]):
                assert abs(a - b) <= 1e-5 * abs(a), (ckpt, resident[r][0], resharded[r][0])
            for k, v in resident[r][1].items():
                # CPU float sums are not bitwise reproducible across runs, and Adam's first updates are about
                # lr * sign(g): a last-bit difference in a near-zero gradient moves that weight by up to 2 lr.
                # So the whole tensor is compared, with a bound (2e-3) far below what one stale or wrong
                # gather would cause (one step's update is a few percent of these weights' norm)
                rel = ((v - resharded[r][1][k]).norm() / v.norm()).item()
                assert rel < 2e-3, (ckpt, k, rel)


def _train_hsdp(rank, world, port, hsdp, reshard=False):
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.optim import FlatAdamW

    initialize_process_group()
    shard_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
    rep_groups = [dist.new_group([0, 2]), dist.new_group([1, 3])]
    model = build_qwen3("mvp/qwen3-tiny", seed=4, vocab_size=256, hidden_size=128, intermediate_size=256,
                        num_attention_heads=2, num_key_value_heads=1, num_hidden_layers=2)
    if hsdp:
        fsdp = NativeFSDP(model, group=shard_groups[rank // 2], device=torch.device("cpu"),
                          param_dtype=torch.float32, replicate_group=rep_groups[rank % 2],
                          reshard_after_forward=reshard)
        assert fsdp.world == 2 and fsdp.rep_world == 2
    else:
        fsdp = NativeFSDP(model, group=dist.group.WORLD, device=torch.device("cpu"), param_dtype=torch.float32)
    opt = FlatAdamW(fsdp, lr=1e-3, weight_decay=0.1)
    g = torch.Generator().manual_seed(77)
    losses = []
    for _ in range(4):
        x = torch.randint(0, 256, (4, 40), generator=g)[rank:rank + 1]
        loss = fsdp(input_ids=x, labels=x)["loss"].sum() / 39
        loss.backward()
        fsdp.clip_grad_norm_(1.0)
        opt.step()
        t = loss.detach().clone()
        dist.all_reduce(t)
        losses.append(float(t) / world)
    full = fsdp.checkpoint_state_dict(full=True)
    return losses, {k: v.clone() for k, v in full.items() if "layers.1." in k}


@pytest.mark.parametrize("reshard", [False, True])
def test_hsdp_matches_flat_sharding(reshard):
    """Replicate x shard (2 x 2) with gradient shards averaged over the replicas equals sharding over all 4,
    with resident weights and with weights resharded after each use (gathered within the shard group)."""
    flat = spawn_workers(_train_hsdp, 4, False, timeout=300)
    hsdp = spawn_workers(_train_hsdp, 4, True, reshard, timeout=300)
    for (lf, wf), (lh, wh) in zip(flat, hsdp):
        for a, b in zip(lf, lh):
            assert abs(a - b) <= 1e-5 * abs(a), (lf, lh)
        for k, v in wf.items():
            # fp32 sums in another order; Adam turns last-bit differences of near-zero gradients into
            # lr-sized weight differences (see the resharding test for the bound)
            assert ((v - wh[k]).norm() / v.norm()).item() < 2e-3, (k, ((v - wh[k]).norm() / v.norm()).item())
