"""Ring / Ulysses context parallelism on 2 GPUs (NCCL) against single-GPU attention of the whole row."""

import pytest
import torch

from mvp_engine.testing import spawn_workers

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 CUDA devices")


def _inputs(T, Hq, Hkv, device):
    g = torch.Generator().manual_seed(5)
    q = torch.randn(T, Hq, 128, generator=g).bfloat16().to(device)
    k = torch.randn(T, Hkv, 128, generator=g).bfloat16().to(device)
    v = torch.randn(T, Hkv, 128, generator=g).bfloat16().to(device)
    do = torch.randn(T, Hq, 128, generator=g).bfloat16().to(device)
    lens = [700, 1500, 300, 2500, T - 5000]
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=device)
    return q, k, v, do, cu


def _worker(rank, world, port, impl, T):
    import os

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import PackedContext
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.context import ContextParallel

    initialize_process_group()
    dev = torch.device("cuda", torch.cuda.current_device())
    q, k, v, do, cu = _inputs(T, 16, 8, dev)
    cp = ContextParallel(dist.group.WORLD, impl=impl)
    idx = cp.local_indices(T).to(dev)
    ql, kl, vl = (t[idx].clone().requires_grad_() for t in (q, k, v))
    ctx = PackedContext(torch.zeros(1, len(idx), dtype=torch.long, device=dev), cu,
                        int((cu[1:] - cu[:-1]).max()), None, cp=cp)
    o = cp.attention(ql, kl, vl, ctx, 128**-0.5)
    o.backward(do[idx])
    torch.cuda.synchronize()
    _ext.check_status(dev)
    res = [t.detach().cpu() for t in (idx, o, ql.grad, kl.grad, vl.grad)]
    dist.barrier()
    return res


@two_gpus
@pytest.mark.parametrize("impl", ["ring", "ulysses"])
def test_context_parallel_two_gpus(impl):
    from mvp_engine.ops.attention import flash_attn_varlen

    T = 8192
    q, k, v, do, cu = _inputs(T, 16, 8, "cuda")
    qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
    ref = flash_attn_varlen(qq, kk, vv, cu, int((cu[1:] - cu[:-1]).max()), causal=True, softmax_scale=128**-0.5)
    ref.backward(do)
    out = spawn_workers(_worker, 2, impl, T, timeout=300)
    o = torch.zeros_like(q).cpu()
    g = [torch.zeros_like(t).cpu() for t in (q, k, v)]
    for idx, ol, gq, gk, gv in out:
        o[idx], g[0][idx], g[1][idx], g[2][idx] = ol, gq, gk, gv

    def rel(a, b):
        return ((a.float() - b.float().cpu()).norm() / b.float().norm().cpu()).item()

    assert rel(o, ref.detach()) < 1e-2
    for a, b in zip(g, (qq.grad, kk.grad, vv.grad)):
        assert rel(a, b) < 2e-2
