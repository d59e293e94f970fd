"""Pull reduce-scatter over NVLink peer memory (symmetric buffers) and its bounded waits."""

import pytest
import torch

from mvp_engine.testing import spawn_workers

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 CUDA devices")


@cuda
def test_peer_wait_runs_out_and_reports_status():
    """A peer that never publishes: the kernel gives up after its bound, sets kTimeoutPeer, reads no
    peer memory, and the context stays usable."""
    from mvp_engine import ops
    from mvp_engine.ops import _ext

    buf = torch.zeros(1024, device="cuda")
    other = torch.zeros(1024, device="cuda")  # stands in for the absent peer's buffer (never read)
    slots = torch.zeros(8, dtype=torch.int64, device="cuda")
    other_slots = torch.zeros(8, dtype=torch.int64, device="cuda")
    out = torch.empty(512, device="cuda")
    _ext.check_status(0)
    ops.peer_reduce_scatter([buf.data_ptr(), other.data_ptr()], [slots.data_ptr(), other_slots.data_ptr()],
                            slots.data_ptr(), 0, 0, 512, 1, out, timeout_s=0.3)
    torch.cuda.synchronize()
    assert int(_ext.status_buffer(0)[0]) == 5  # kTimeoutPeer
    with pytest.raises(RuntimeError):
        _ext.check_status(0)
    assert int(other_slots[0]) == 1  # this rank still published its own readiness
    x = torch.ones(1000, device="cuda")
    assert float(x.sum()) == 1000.0


def _rs_worker(rank, world, port):
    import os

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm

    from mvp_engine import ops
    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.ops import _ext

    initialize_process_group()
    dev = torch.device("cuda", torch.cuda.current_device())
    n = 2 * 4096 * world
    buf = symm.empty(n, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    buf.copy_(torch.randn(n, generator=g, device=dev))
    slots = symm.empty(8, dtype=torch.int64, device=dev)
    slots.zero_()
    torch.cuda.synchronize()
    hb, hs = symm.rendezvous(buf, dist.group.WORLD), symm.rendezvous(slots, dist.group.WORLD)
    hs.barrier()
    shard = 4096
    outs = []
    for unit, seq in ((0, 1), (1, 2)):
        out = torch.empty(shard, device=dev)
        ssq = torch.zeros(1, device=dev)
        ops.peer_reduce_scatter([int(p) for p in hb.buffer_ptrs], [int(p) for p in hs.buffer_ptrs],
                                slots.data_ptr(), rank, unit * shard * world, shard, seq, out, scale=0.5, sumsq=ssq)
        outs.append((out, ssq))
    ops.peer_barrier([int(p) for p in hs.buffer_ptrs], slots.data_ptr(), rank, 3)
    torch.cuda.synchronize()
    _ext.check_status(dev)
    full = torch.empty(world, n, device=dev)
    dist.all_gather_into_tensor(full, buf)
    res = []
    for unit, (out, ssq) in enumerate(outs):
        lo = unit * shard * world + rank * shard
        ref = 0.5 * full[:, lo:lo + shard].sum(0)
        res.append(((out - ref).abs().max().item(), abs(ssq.item() - float(ref.pow(2).sum())) / float(ref.pow(2).sum())))
    dist.barrier()
    return res


@two_gpus
def test_peer_reduce_scatter_two_gpus():
    for res in spawn_workers(_rs_worker, 2, timeout=300):
        for err, ssq_rel in res:
            assert err < 1e-5 and ssq_rel < 1e-4


# Two runs compared after AdamW steps must add the same numbers in the same order: Adam's first update
# is about lr * sign(g), so a last-bit difference in a near-zero gradient becomes an lr-sized weight
# difference.  The weight-gradient GEMM's split-k tail adds its pieces in no fixed order, so the strict
# comparisons run it on whole tiles only (MVP_GEMM_STREAMK=0); one reshard variant keeps it on and is
# compared with a tolerance that allows for the order.
_SPLIT_TOL = 5e-3


def _fsdp_worker(rank, world, port, comm):
    import os

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["MVP_GEMM_STREAMK"] = "0"
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.optim import FlatAdamW

    initialize_process_group()
    dev = torch.device("cuda", torch.cuda.current_device())
    model = build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=512, num_hidden_layers=2, device="meta")
    fsdp = NativeFSDP(model, group=dist.group.WORLD, device=dev, param_dtype=torch.bfloat16, comm=comm)
    assert (fsdp._peer is not None) == (comm == "fused")
    opt = FlatAdamW(fsdp, lr=1e-3)
    g = torch.Generator().manual_seed(7 + rank)
    T = 1024
    cu = torch.tensor([0, 300, T], dtype=torch.int32, device=dev)
    losses = []
    for _ in range(2):
        ids = torch.randint(0, 512, (1, T), generator=g).to(dev)
        out = fsdp(input_ids=ids, labels=ids, cu_seq_lens_q=cu, max_length_q=724)
        loss = out["loss"].sum() / T
        loss.backward()
        gn = fsdp.clip_grad_norm_(1.0)
        shards = [s.detach().float().cpu().clone() for s in fsdp.grad_shards()]
        opt.step()
        losses.append((float(loss), float(gn)))
    torch.cuda.synchronize()
    _ext.check_status(dev)
    dist.barrier()
    return losses, shards


@two_gpus
def test_native_fsdp_peer_reduce_scatter_matches_nccl():
    fused = spawn_workers(_fsdp_worker, 2, "fused", timeout=300)
    nccl = spawn_workers(_fsdp_worker, 2, "nccl", timeout=300)
    for (lf, sf), (ln, sn) in zip(fused, nccl):
        for (a, ga), (b, gb) in zip(lf, ln):
            assert abs(a - b) < 1e-3 * abs(b) and abs(ga - gb) < 1e-3 * abs(gb)
        for x, y in zip(sf, sn):
            assert ((x - y).norm() / (y.norm() + 1e-12)).item() < 1e-4


def _reshard_worker(rank, world, port, comm, reshard, ckpt, gather="gemm", split_k=False):
    import os

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["MVP_GEMM_STREAMK"] = "1" if split_k else "0"
    # gemm: every pull rides in copy CTAs of the next GEMM (threshold 0 so the tiny model's GEMMs carry
    # it); kernel: stand-alone pull kernel on the comm stream
    os.environ["MVP_FSDP_GATHER"] = gather
    os.environ["MVP_FSDP_GATHER_MIN_MNK"] = "0"
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.optim import FlatAdamW

    initialize_process_group()
    dev = torch.device("cuda", torch.cuda.current_device())
    model = build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=512, num_hidden_layers=4, device="meta")
    if ckpt:
        model.gradient_checkpointing_enable({"num_layers": 2})
    fsdp = NativeFSDP(model, group=dist.group.WORLD, device=dev, param_dtype=torch.bfloat16, comm=comm,
                      reshard_after_forward=reshard)
    assert sum(u.resharded for u in fsdp.units) == (4 if reshard else 0)
    assert (fsdp._wpeer is not None) == (reshard and comm == "fused")
    from mvp_engine import ops

    carried = [0]
    real = ops._carry_pending_gather

    def counting(*a, **k):
        launched = real(*a, **k)
        carried[0] += int(launched)
        return launched

    ops._carry_pending_gather = counting
    opt = FlatAdamW(fsdp, lr=1e-3)
    g = torch.Generator().manual_seed(11 + rank)
    T = 1024
    cu = torch.tensor([0, 300, T], dtype=torch.int32, device=dev)
    losses = []
    for _ in range(3):
        total = 0.0
        for micro in range(2):
            ids = torch.randint(0, 512, (1, T), generator=g).to(dev)
            fsdp.set_requires_gradient_sync(micro == 1)
            out = fsdp(input_ids=ids, labels=ids, cu_seq_lens_q=cu, max_length_q=724)
            loss = out["loss"].sum() / T
            loss.backward()
            total += float(loss.detach())
        gn = fsdp.clip_grad_norm_(1.0)
        opt.step()
        losses.append((total, float(gn)))
    torch.cuda.synchronize()
    _ext.check_status(dev)
    sd = fsdp.checkpoint_state_dict(full=True)
    dist.barrier()
    if reshard and comm == "fused" and gather == "gemm":
        assert carried[0] > 0, "no GEMM carried a gather"
    return losses, {k: v.float().clone() for k, v in sd.items() if "layers.3." in k}


@two_gpus
@pytest.mark.parametrize("ckpt", [False, True])
def test_resharded_weights_peer_pull_matches_resident(ckpt):
    """FSDP parameter gather by peer pull (weights resharded after each use, gathered again for backward and
    recomputation) -- carried by GEMM copy CTAs, or as a stand-alone kernel -- against NCCL all-gathers
    and against resident weights: same losses, norms and weights."""
    resident = spawn_workers(_reshard_worker, 2, "nccl", False, ckpt, timeout=300)
    in_gemm = spawn_workers(_reshard_worker, 2, "fused", True, ckpt, "gemm", timeout=300)
    pulled = spawn_workers(_reshard_worker, 2, "fused", True, ckpt, "kernel", timeout=300)
    gathered = spawn_workers(_reshard_worker, 2, "nccl", True, ckpt, timeout=300)
    # gathers carried by GEMMs whose weight gradients use the split-k tail (the production setting)
    in_gemm_split = spawn_workers(_reshard_worker, 2, "fused", True, ckpt, "gemm", True, timeout=300)
    for variant, tol in ((in_gemm, 1e-4), (pulled, 1e-4), (gathered, 1e-4), (in_gemm_split, _SPLIT_TOL)):
        for (lv, wv), (lr, wr) in zip(variant, resident):
            for (a, ga), (b, gb) in zip(lv, lr):
                assert abs(a - b) <= 1e-3 * abs(b) and abs(ga - gb) <= 1e-3 * abs(gb), (lv, lr)
            for k, v in wr.items():
                assert ((wv[k] - v).norm() / (v.norm() + 1e-12)).item() < tol, k
