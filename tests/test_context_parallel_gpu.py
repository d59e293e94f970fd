"""Ring / Ulysses context parallelism on 2 GPUs against single-GPU attention of the whole row.

``fused`` selects the NVLink peer-memory kernels (ring: K/V pulled by copy CTAs of the attention
kernel, dK/dV partials written into the owner's slots); otherwise the collectives are NCCL calls.
"""

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


def _worker(rank, world, port, impl, T, fused=False):
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
    cp = ContextParallel(dist.group.WORLD, impl=impl, fused=fused)
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
@pytest.mark.parametrize("impl,fused", [("ring", False), ("ulysses", False), ("ring", True)])
def test_context_parallel_two_gpus(impl, fused):
    from mvp_engine.ops.attention import flash_attn_varlen

    T = 8192
    q, k, v, do, cu = _inputs(T, 16, 8, "cuda")
    qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
    ref = flash_attn_varlen(qq, kk, vv, cu, int((cu[1:] - cu[:-1]).max()), causal=True, softmax_scale=128**-0.5)
    ref.backward(do)
    out = spawn_workers(_worker, 2, impl, T, fused, timeout=300)
    o = torch.zeros_like(q).cpu()
    g = [torch.zeros_like(t).cpu() for t in (q, k, v)]
    for idx, ol, gq, gk, gv in out:
        o[idx], g[0][idx], g[1][idx], g[2][idx] = ol, gq, gk, gv

    def rel(a, b):
        return ((a.float() - b.float().cpu()).norm() / b.float().norm().cpu()).item()

    assert rel(o, ref.detach()) < 1e-2
    for a, b in zip(g, (qq.grad, kk.grad, vv.grad)):
        assert rel(a, b) < 2e-2


def _layer_worker(rank, world, port, fused, T):
    import os

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist

    from mvp_engine import ops
    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import PackedContext, Qwen3DecoderLayer, load_qwen3_config, positions_from_cu_seqlens
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.context import ContextParallel

    initialize_process_group()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = load_qwen3_config("mvp/qwen3-tiny", hidden_size=512, intermediate_size=1024, num_attention_heads=4,
                            num_key_value_heads=2)
    layer = Qwen3DecoderLayer(cfg, 0).to(dev)
    g = torch.Generator().manual_seed(11)
    with torch.no_grad():
        for name, p in sorted(layer.named_parameters()):
            base = 1.0 if "norm" in name else 0.0
            p.copy_((base + 0.05 * torch.randn(p.shape, generator=g)).to(dev))
    x = torch.randn(T, 512, generator=g).bfloat16().to(dev)
    dy1 = torch.randn(T, 512, generator=g).bfloat16().to(dev)
    dy2 = torch.randn(T, 512, generator=g).bfloat16().to(dev)
    lens = [700, 1500, 300, T - 2500]
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=dev)
    cp = ContextParallel(dist.group.WORLD, impl="ulysses", fused=fused)
    idx = cp.local_indices(T).to(dev)
    xl = x[idx].clone().requires_grad_()
    pos = positions_from_cu_seqlens(cu, T)[idx].view(1, -1).to(torch.int32)
    rope = ops.RopeCache(128, cfg.rope_theta, max_positions=4096)
    ctx = PackedContext(pos, cu, max(lens), rope, cp=cp)
    out, res = layer(xl, None, ctx)
    torch.autograd.backward([out, res], [dy1[idx], dy2[idx]])
    torch.cuda.synchronize()
    _ext.check_status(dev)
    grads = {n: p.grad.detach().float().cpu() for n, p in layer.named_parameters() if p.grad is not None}
    res_ = [idx.cpu(), out.detach().cpu(), res.detach().cpu(), xl.grad.detach().cpu(), grads]
    dist.barrier()
    return res_


@two_gpus
def test_ulysses_fused_layer_two_gpus():
    """A decoder layer under Ulysses with the all-to-alls fused into the GEMM / attention / norm kernels
    against the same layer with NCCL all-to-alls: outputs, input gradients and weight gradients summed
    over the ranks (the fused path gives each rank the norm-weight gradient of its heads instead of its
    tokens; the sums agree)."""
    T = 4096
    ref = spawn_workers(_layer_worker, 2, False, T, timeout=300)
    fused = spawn_workers(_layer_worker, 2, True, T, timeout=300)

    def rel(a, b):
        return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()

    for (i0, o0, r0, g0, _), (i1, o1, r1, g1, _) in zip(ref, fused):
        assert torch.equal(i0, i1)
        assert rel(o1, o0) < 2e-2
        assert rel(r1, r0) < 2e-2
        assert rel(g1, g0) < 3e-2
    names = ref[0][4].keys()
    assert set(names) == set(fused[0][4].keys())
    for n in names:
        a = sum(w[4][n] for w in fused)
        b = sum(w[4][n] for w in ref)
        assert rel(a, b) < 3e-2, n
