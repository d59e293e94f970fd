"""Vision-tower kernels (LayerNorm, bias + GELU, vision RoPE) against plain PyTorch fp32 references."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _ops():
    from mvp_engine import ops

    return ops


def _rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@cuda
@pytest.mark.parametrize("rows,H", [(1, 192), (333, 1152), (4100, 1152), (517, 4608)])
def test_layer_norm(rows, H):
    ops = _ops()
    torch.manual_seed(0)
    x = (torch.randn(rows, H, device="cuda") * 2 + 0.5).bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_()
    b = (0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_()
    y = ops.layer_norm(x, w, b, 1e-6)
    xf, wf, bf = (t.detach().float().requires_grad_() for t in (x, w, b))
    ref = F.layer_norm(xf, (H,), wf, bf, 1e-6)
    assert _rel_err(y, ref) < 8e-3
    g = torch.randn(rows, H, device="cuda").bfloat16()
    y.backward(g)
    ref.backward(g.float())
    assert _rel_err(x.grad, xf.grad) < 1e-2
    assert _rel_err(w.grad, wf.grad) < 1e-2
    assert _rel_err(b.grad, bf.grad) < 1e-2


@cuda
def test_layer_norm_grad_accumulators():
    """With fp32 accumulators attached, the kernels add the weight / bias gradients into them."""
    ops = _ops()
    torch.manual_seed(1)
    rows, H = 700, 1152
    x = torch.randn(rows, H, device="cuda").bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_()
    b = torch.zeros(H, device="cuda").bfloat16().requires_grad_()
    w._mvp_grad_acc = torch.ones(H, device="cuda")
    b._mvp_grad_acc = torch.ones(H, device="cuda")
    g = torch.randn(rows, H, device="cuda").bfloat16()
    ops.layer_norm(x, w, b, 1e-6).backward(g)
    assert w.grad is None and b.grad is None
    xf, wf, bf = (t.detach().float().requires_grad_() for t in (x, w, b))
    F.layer_norm(xf, (H,), wf, bf, 1e-6).backward(g.float())
    assert _rel_err(w._mvp_grad_acc - 1, wf.grad) < 1e-2
    assert _rel_err(b._mvp_grad_acc - 1, bf.grad) < 1e-2


@cuda
@pytest.mark.parametrize("approximate", ["tanh", "none"])
@pytest.mark.parametrize("rows,Fd", [(1, 768), (1000, 4304), (257, 4608)])
def test_bias_gelu(approximate, rows, Fd):
    ops = _ops()
    torch.manual_seed(0)
    x = (torch.randn(rows, Fd, device="cuda") * 2).bfloat16().requires_grad_()
    b = (0.5 * torch.randn(Fd, device="cuda")).bfloat16().requires_grad_()
    y = ops.bias_gelu(x, b, approximate)
    xf, bf = (t.detach().float().requires_grad_() for t in (x, b))
    ref = F.gelu(xf + bf, approximate=approximate)
    assert _rel_err(y, ref) < 8e-3
    g = torch.randn(rows, Fd, device="cuda").bfloat16()
    y.backward(g)
    ref.backward(g.float())
    assert _rel_err(x.grad, xf.grad) < 1e-2
    assert _rel_err(b.grad, bf.grad) < 1e-2


@cuda
@pytest.mark.parametrize("rows,H", [(1, 1152), (3000, 1152), (257, 4096)])
def test_bias_residual(rows, H):
    ops = _ops()
    torch.manual_seed(0)
    y = torch.randn(rows, H, device="cuda").bfloat16().requires_grad_()
    x = torch.randn(rows, H, device="cuda").bfloat16().requires_grad_()
    b = torch.randn(H, device="cuda").bfloat16().requires_grad_()
    out = ops.bias_residual(y, b, x)
    yf, xf, bf = (t.detach().float().requires_grad_() for t in (y, x, b))
    ref = xf + (yf + bf)
    assert _rel_err(out, ref) < 8e-3
    g = torch.randn(rows, H, device="cuda").bfloat16()
    out.backward(g)
    ref.backward(g.float())
    assert _rel_err(x.grad, xf.grad) < 1e-2 and _rel_err(y.grad, yf.grad) < 1e-2
    assert _rel_err(b.grad, bf.grad) < 1e-2
    b2 = b.detach().clone().requires_grad_()
    b2._mvp_grad_acc = torch.ones(H, device="cuda")
    ops.bias_residual(y.detach(), b2, x.detach()).backward(g)
    assert b2.grad is None and _rel_err(b2._mvp_grad_acc - 1, bf.grad) < 1e-2


@cuda
@pytest.mark.parametrize("N,nh,D", [(1, 16, 72), (1000, 16, 72), (300, 3, 64), (50, 4, 32)])
def test_vision_rope_pad(N, nh, D):
    ops = _ops()
    torch.manual_seed(0)
    qkv = torch.randn(N, 3 * nh * D, device="cuda").bfloat16().requires_grad_()
    ang = torch.rand(N, D // 2, device="cuda") * 50
    q, k, v = ops.vision_rope_pad(qkv, nh, ang.cos(), ang.sin(), 128)
    assert q.shape == (N, nh, 128)
    t = qkv.detach().float().view(N, 3, nh, D).requires_grad_()
    c = torch.cat([ang.cos(), ang.cos()], -1).unsqueeze(1)
    s = torch.cat([ang.sin(), ang.sin()], -1).unsqueeze(1)

    def rot(x):
        a, bb = x.chunk(2, dim=-1)
        return torch.cat((-bb, a), -1)

    rq = t[:, 0] * c + rot(t[:, 0]) * s
    rk = t[:, 1] * c + rot(t[:, 1]) * s
    rv = t[:, 2]
    for out, ref in ((q, rq), (k, rk), (v, rv)):
        assert _rel_err(out[..., :D], ref) < 8e-3
        assert out[..., D:].abs().max().item() == 0
    gq, gk, gv = (torch.randn(N, nh, 128, device="cuda").bfloat16() for _ in range(3))
    (q.float() * gq.float()).sum().add((k.float() * gk.float()).sum()).add((v.float() * gv.float()).sum()).backward()
    ((rq * gq[..., :D].float()).sum() + (rk * gk[..., :D].float()).sum() + (rv * gv[..., :D].float()).sum()).backward()
    assert _rel_err(qkv.grad, t.grad.reshape(N, -1)) < 1e-2


@cuda
@pytest.mark.parametrize("D", [72, 80])
def test_vision_rope_pad_with_fused_bias(D):
    """qkv bias added inside the RoPE kernel: forward and both gradients against fp32 (bias + rotation)."""
    ops = _ops()
    torch.manual_seed(1)
    N, nh = 777, 4
    qkv = torch.randn(N, 3 * nh * D, device="cuda").bfloat16().requires_grad_()
    b = (0.5 * torch.randn(3 * nh * D, device="cuda")).bfloat16().requires_grad_()
    ang = torch.rand(N, D // 2, device="cuda") * 50
    q, k, v = ops.vision_rope_pad(qkv, nh, ang.cos(), ang.sin(), 128, bias=b)
    tq = qkv.detach().float().requires_grad_()
    tb = b.detach().float().requires_grad_()
    t = (tq + tb).view(N, 3, nh, D)
    c = torch.cat([ang.cos(), ang.cos()], -1).unsqueeze(1)
    s = torch.cat([ang.sin(), ang.sin()], -1).unsqueeze(1)

    def rot(x):
        a, bb = x.chunk(2, dim=-1)
        return torch.cat((-bb, a), -1)

    refs = (t[:, 0] * c + rot(t[:, 0]) * s, t[:, 1] * c + rot(t[:, 1]) * s, t[:, 2])
    for out, ref in zip((q, k, v), refs):
        assert _rel_err(out[..., :D], ref) < 8e-3
    gs = [torch.randn(N, nh, 128, device="cuda").bfloat16() for _ in range(3)]
    sum((o.float() * g.float()).sum() for o, g in zip((q, k, v), gs)).backward()
    sum((r * g[..., :D].float()).sum() for r, g in zip(refs, gs)).backward()
    assert _rel_err(qkv.grad, tq.grad) < 1e-2
    assert _rel_err(b.grad, tb.grad) < 1e-2


@cuda
def test_vision_block_matches_eager():
    """One Qwen3-VL vision block on the native kernels against the same block in fp32 eager math."""
    from mvp_engine.models import qwen3_vl as vl

    torch.manual_seed(0)
    c = vl.Qwen3VLVisionConfig(hidden_size=1152, num_heads=16, intermediate_size=4304)
    blk = vl.Qwen3VLVisionBlock(c)
    for p in blk.parameters():
        torch.nn.init.normal_(p, std=0.05)
    for ln in (blk.norm1, blk.norm2):
        torch.nn.init.normal_(ln.weight, mean=1.0, std=0.1)
    N = 600
    cu = torch.tensor([0, 256, 600], dtype=torch.int32)
    ang = torch.rand(N, 36) * 30
    x = torch.randn(N, 1152)
    ref = blk(x, cu, 344, ang.cos(), ang.sin())  # CPU fp32: eager math
    blk = blk.cuda().bfloat16()
    angc = ang.cuda()
    out = blk(x.cuda().bfloat16(), cu.cuda(), 344, angc.cos(), angc.sin())
    assert _rel_err(out.cpu(), ref) < 2e-2


@cuda
def test_qwen3_vl_vision_tower_native_matches_fp32():
    """Tiny Qwen3-VL vision tower: bf16 on the native kernels vs fp32 eager on CPU, outputs and gradients."""
    from mvp_engine.models.qwen3_vl import build_qwen3_vl

    torch.manual_seed(0)
    vis = build_qwen3_vl("mvp/qwen3-vl-tiny", seed=0).model.visual
    vc = vis.config
    grids = torch.tensor([[1, 4, 4], [1, 8, 12]])
    n = int(sum(t * h * w for t, h, w in grids.tolist()))
    pix = torch.randn(n, vc.in_channels * vc.temporal_patch_size * vc.patch_size ** 2)
    ref, ref_deep = vis(pix, grids)
    G = torch.randn_like(ref)
    (ref * G).sum().backward()
    ref_grads = {k: p.grad.clone() for k, p in vis.named_parameters() if p.grad is not None}
    vis.zero_grad(set_to_none=True)
    vis = vis.cuda()
    out, deep = vis(pix.cuda(), grids, dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    assert _rel_err(out.cpu(), ref) < 3e-2
    for a, b in zip(deep, ref_deep):
        assert _rel_err(a.cpu(), b) < 3e-2
    (out.float() * G.cuda()).sum().backward()
    for name in ("blocks.0.norm1.weight", "blocks.0.norm1.bias", "blocks.1.mlp.linear_fc1.bias",
                 "blocks.2.attn.qkv.weight", "merger.linear_fc1.bias", "patch_embed.proj.weight"):
        got = dict(vis.named_parameters())[name].grad
        assert got is not None, name
        assert _rel_err(got.cpu(), ref_grads[name]) < 5e-2, name


@cuda
def test_split_linear_fp32_accuracy_forward_backward():
    """Patch-embed GEMM in fp32 accuracy (hi/lo bf16 splits on tcgen05): forward, dX and dW against fp64."""
    from mvp_engine.models.qwen3_vl import linear_fp32_accurate

    torch.manual_seed(21)
    x = torch.randn(3000, 1536, device="cuda", dtype=torch.float32).requires_grad_()
    w = (0.02 * torch.randn(1152, 1536, device="cuda")).requires_grad_()
    b = (0.1 * torch.randn(1152, device="cuda")).requires_grad_()
    y = linear_fp32_accurate(x, w, b)
    g = torch.randn_like(y)
    y.backward(g)
    xd, wd, bd = (t.detach().double().requires_grad_() for t in (x, w, b))
    yd = xd @ wd.t() + bd
    yd.backward(g.double())
    for got, ref in ((y, yd), (x.grad, xd.grad), (w.grad, wd.grad), (b.grad, bd.grad)):
        rel = ((got.double() - ref).norm() / ref.norm()).item()
        assert rel < 1e-4, rel
