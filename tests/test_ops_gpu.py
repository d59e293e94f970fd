"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _ops():
    from mvp_engine import ops

    return ops


def _rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


GEMM_SHAPES = [
    (128, 256, 64),
    (256, 512, 128),
    (200, 300, 72),
    (1, 8, 8),
    (1000, 1000, 1000),
    (129, 257, 520),
    (1024, 3072, 4096),
    (520, 776, 136),      # two-SM 256 x 256 tiles with ragged M / N tails
    (2048, 4096, 8192),
]


@cuda
@pytest.mark.parametrize("shape", GEMM_SHAPES)
@pytest.mark.parametrize("majors", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_majors(shape, majors):
    ops = _ops()
    M, N, K = shape
    a_mn, b_mn = majors
    torch.manual_seed(0)
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    a_in = A.t().contiguous() if a_mn else A
    b_in = B.t().contiguous() if b_mn else B
    if a_mn and (M % 8):
        pytest.skip("MN-major A needs M % 8 == 0 for the TMA row stride")
    if b_mn and (N % 8):
        pytest.skip("MN-major B needs N % 8 == 0 for the TMA row stride")
    ref = A.float() @ B.float().t()
    out = ops.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _rel_err(out, ref) < 1e-5, (shape, majors)
    out16 = ops.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn)
    assert _rel_err(out16, ref) < 8e-3
    acc = torch.ones(M, N, device="cuda")
    ops.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out=acc, accumulate=True)
    assert _rel_err(acc, ref + 1) < 1e-5
    from mvp_engine.ops import _ext

    _ext.check_status()


@cuda
@pytest.mark.parametrize(
    "shape",
    [
        (6144, 4096, 8192),  # QKV weight gradient: 384 tiles, a 14-tile last wave split over k
        (4096, 4096, 1000),  # 256 tiles, ragged k (16 blocks, the last one partial)
        (768, 1024, 4096),   # 12 tiles, fewer than the clusters: every tile split
        (1000, 776, 2048),   # ragged M / N edges in split tiles (scalar reduction path)
    ],
)
def test_gemm_accumulate_split_k_tail(shape):
    """Weight-gradient GEMM into an fp32 accumulator (dW += dY^T X, both operands MN-major), where the
    k-blocks of the last, partial wave of tiles are spread over all clusters and added by reductions:
    two accumulations in a row onto a non-zero buffer must equal the fp32 product twice plus the
    starting values."""
    ops = _ops()
    M, N, K = shape
    torch.manual_seed(3)
    dy = torch.randn(K, M, device="cuda").bfloat16()  # [tokens, out features]
    x = torch.randn(K, N, device="cuda").bfloat16()   # [tokens, in features]
    ref = dy.float().t() @ x.float()
    start = torch.randn(M, N, device="cuda")
    acc = start.clone()
    ops.gemm(dy, x, a_mn=True, b_mn=True, out=acc, accumulate=True)
    torch.cuda.synchronize()
    assert _rel_err(acc - start, ref) < 1e-5, shape
    ops.gemm(dy, x, a_mn=True, b_mn=True, out=acc, accumulate=True)
    torch.cuda.synchronize()
    assert _rel_err(acc - start, 2 * ref) < 1e-5, shape
    from mvp_engine.ops import _ext

    _ext.check_status()


@cuda
def test_gemm_strided_views():
    ops = _ops()
    torch.manual_seed(1)
    big = torch.randn(512, 1024, device="cuda").bfloat16()
    A = big[:, 128:640]  # row stride 1024
    W = torch.randn(384, 512, device="cuda").bfloat16()
    out = ops.gemm(A, W, out_dtype=torch.float32)
    ref = A.float() @ W.float().t()
    assert _rel_err(out, ref) < 1e-5


@cuda
def test_linear_autograd():
    ops = _ops()
    torch.manual_seed(2)
    x = torch.randn(4, 96, 256, device="cuda").bfloat16().requires_grad_()
    w = torch.randn(384, 256, device="cuda").bfloat16().requires_grad_()
    y = ops.linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xf = x.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    yf = xf @ wf.t()
    yf.backward(g.float())
    assert _rel_err(y, yf) < 8e-3
    assert _rel_err(x.grad, xf.grad) < 8e-3
    assert _rel_err(w.grad, wf.grad) < 8e-3
    # accumulate-into-buffer path
    w2 = w.detach().clone()
    w2._mvp_grad_acc = torch.zeros(w2.shape, device="cuda")
    x2 = x.detach().clone().requires_grad_()
    ops.linear(x2, w2).backward(g)
    ops.linear(x2, w2).backward(g)
    assert _rel_err(w2._mvp_grad_acc, 2 * wf.grad) < 1e-4


@cuda
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm(with_res):
    ops = _ops()
    torch.manual_seed(3)
    T, H = 333, 4096
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    r = torch.randn(T, H, device="cuda").bfloat16().requires_grad_() if with_res else None
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_()
    y, h = ops.rms_norm(x, w, 1e-6, residual=r)
    gy = torch.randn_like(y)
    gh = torch.randn_like(h) if with_res else None
    torch.autograd.backward([y] + ([h] if with_res else []), [gy] + ([gh] if with_res else []))

    xf = x.detach().float().requires_grad_()
    rf = r.detach().float().requires_grad_() if with_res else None
    wf = w.detach().float().requires_grad_()
    hf = xf + rf if with_res else xf
    yf = wf * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6))
    torch.autograd.backward([yf] + ([hf] if with_res else []), [gy.float()] + ([gh.float()] if with_res else []))
    assert _rel_err(y, yf) < 1e-2
    assert _rel_err(x.grad, xf.grad) < 1e-2
    assert _rel_err(w.grad, wf.grad) < 1e-2
    if with_res:
        assert _rel_err(r.grad, rf.grad) < 1e-2


@cuda
@pytest.mark.parametrize("with_res", [False, True])
def test_rms_norm_linear_matches_fp32(with_res):
    """The fused norm -> GEMM node (normalised rows recomputed in the backward) against fp32 PyTorch."""
    ops = _ops()
    torch.manual_seed(5)
    T, H, N = 520, 1024, 768
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    r = torch.randn(T, H, device="cuda").bfloat16().requires_grad_() if with_res else None
    wn = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_()
    wl = (0.02 * torch.randn(N, H, device="cuda")).bfloat16().requires_grad_()
    y, h = ops.rms_norm_linear(x, wn, wl, 1e-6, residual=r)
    gy, gh = torch.randn_like(y), torch.randn_like(h)
    torch.autograd.backward([y, h], [gy, gh])

    xf = x.detach().float().requires_grad_()
    rf = r.detach().float().requires_grad_() if with_res else None
    wnf = wn.detach().float().requires_grad_()
    wlf = wl.detach().float().requires_grad_()
    hf = xf + rf if with_res else xf
    yf = (wnf * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6))) @ wlf.t()
    torch.autograd.backward([yf, hf], [gy.float(), gh.float()])
    assert _rel_err(y, yf) < 1e-2
    assert _rel_err(h, hf) < 1e-2
    assert _rel_err(x.grad, xf.grad) < 1e-2
    assert _rel_err(wn.grad, wnf.grad) < 1e-2
    assert _rel_err(wl.grad, wlf.grad) < 1e-2
    if with_res:
        assert _rel_err(r.grad, rf.grad) < 1e-2


@cuda
@pytest.mark.parametrize("mrope", [None, [24, 20, 20]])
def test_qk_norm_rope(mrope):
    ops = _ops()
    torch.manual_seed(4)
    T, Hq, Hkv, D = 300, 8, 2, 128
    cache = ops.RopeCache(D, 1e6, mrope_section=mrope, max_positions=4096)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda").bfloat16().requires_grad_()
    wq = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16().requires_grad_()
    wk = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16().requires_grad_()
    A = 3 if mrope else 1
    pos = torch.randint(0, 3000, (A, T), device="cuda")
    q, k = ops.qk_norm_rope(qkv, Hq, Hkv, wq, wk, pos, cache, 1e-6)
    gq, gk = torch.randn_like(q), torch.randn_like(k)
    torch.autograd.backward([q, k], [gq, gk])

    qkvf = qkv.detach().float().requires_grad_()
    wqf = wq.detach().float().requires_grad_()
    wkf = wk.detach().float().requires_grad_()
    cos, sin = cache.cos_sin(pos, torch.float32)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)

    def norm(x, w):
        return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6))

    def rot(x):
        x1, x2 = x.chunk(2, -1)
        return torch.cat((-x2, x1), -1)

    qf = norm(qkvf[:, : Hq * D].view(T, Hq, D), wqf)
    kf = norm(qkvf[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D), wkf)
    qf = qf * cos + rot(qf) * sin
    kf = kf * cos + rot(kf) * sin
    torch.autograd.backward([qf, kf], [gq.float(), gk.float()])
    assert _rel_err(q, qf) < 1.5e-2
    assert _rel_err(k, kf) < 1.5e-2
    n = (Hq + Hkv) * D
    assert _rel_err(qkv.grad[:, :n], qkvf.grad[:, :n]) < 2e-2
    assert _rel_err(wq.grad, wqf.grad) < 2e-2
    assert _rel_err(wk.grad, wkf.grad) < 2e-2


@cuda
def test_swiglu():
    ops = _ops()
    torch.manual_seed(5)
    gu = torch.randn(257, 2 * 1024, device="cuda").bfloat16().requires_grad_()
    out = ops.swiglu(gu)
    g = torch.randn_like(out)
    out.backward(g)
    guf = gu.detach().float().requires_grad_()
    a, b = guf.chunk(2, -1)
    of = torch.nn.functional.silu(a) * b
    of.backward(g.float())
    assert _rel_err(out, of) < 1e-2
    assert _rel_err(gu.grad, guf.grad) < 1e-2


@cuda
def test_swiglu_linear_matches_fp32():
    """The SwiGLU + down-projection op that recomputes the activation in its backward."""
    ops = _ops()
    torch.manual_seed(9)
    T, F_, H = 512, 768, 512
    gu = torch.randn(T, 2 * F_, device="cuda").bfloat16().requires_grad_()
    w = (torch.randn(H, F_, device="cuda") * 0.05).bfloat16().requires_grad_()
    out = ops.swiglu_linear(gu, w)
    g = torch.randn_like(out)
    out.backward(g)
    guf = gu.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    a, b = guf.chunk(2, -1)
    of = (torch.nn.functional.silu(a) * b) @ wf.t()
    of.backward(g.float())
    assert _rel_err(out, of) < 2e-2
    assert _rel_err(gu.grad, guf.grad) < 2e-2
    assert _rel_err(w.grad, wf.grad) < 2e-2


@cuda
def test_embedding():
    ops = _ops()
    torch.manual_seed(6)
    V, H = 1000, 512
    w = torch.randn(V, H, device="cuda").bfloat16()
    ids = torch.randint(0, V, (3, 77), device="cuda")
    out = ops.embedding(ids, w)
    assert torch.equal(out, w[ids])
    w2 = w.clone().requires_grad_()
    out2 = ops.embedding(ids, w2)
    g = torch.randn_like(out2)
    out2.backward(g)
    ref = torch.zeros(V, H, device="cuda").index_add_(0, ids.reshape(-1), g.reshape(-1, H).float())
    assert _rel_err(w2.grad, ref) < 1e-2


@cuda
def test_fused_linear_ce():
    ops = _ops()
    torch.manual_seed(7)
    T, H, V = 600, 256, 5000
    h = (0.5 * torch.randn(T, H, device="cuda")).bfloat16().requires_grad_()
    w = (0.05 * torch.randn(V, H, device="cuda")).bfloat16().requires_grad_()
    labels = torch.randint(0, V, (T,), device="cuda")
    labels[::7] = -100
    loss = ops.fused_linear_cross_entropy(h, w, labels, chunk_size=256)
    (loss.sum() / 1000).backward()
    hf = h.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    lf = torch.nn.functional.cross_entropy(hf @ wf.t(), labels, ignore_index=-100, reduction="none")
    (lf.sum() / 1000).backward()
    assert _rel_err(loss, lf) < 1e-2
    assert _rel_err(h.grad, hf.grad) < 2e-2
    assert _rel_err(w.grad, wf.grad) < 2e-2


@cuda
def test_fused_linear_ce_backward_in_forward():
    """With the loss gradient promised up front, the LM head's backward runs inside the forward: same loss and
    gradients as the fp32 reference; input gradients also follow a non-uniform per-token gradient."""
    ops = _ops()
    torch.manual_seed(9)
    T, H, V = 600, 256, 5000
    div = 1000.0
    hint = float(torch.tensor(1.0, dtype=torch.float32) / div)
    h = (0.5 * torch.randn(T, H, device="cuda")).bfloat16().requires_grad_()
    w = (0.05 * torch.randn(V, H, device="cuda")).bfloat16().requires_grad_()
    labels = torch.randint(0, V, (T,), device="cuda")
    labels[::7] = -100
    loss = ops.fused_linear_cross_entropy(h, w, labels, chunk_size=256, grad_hint=hint)
    (loss.sum() / div).backward()
    hf = h.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    lf = torch.nn.functional.cross_entropy(hf @ wf.t(), labels, ignore_index=-100, reduction="none")
    (lf.sum() / div).backward()
    assert _rel_err(loss, lf) < 1e-2
    assert _rel_err(h.grad, hf.grad) < 2e-2
    assert _rel_err(w.grad, wf.grad) < 2e-2
    # per-token weights: the input gradient rows are rescaled exactly
    h2 = h.detach().clone().requires_grad_()
    weights = torch.rand(T, device="cuda")
    loss2 = ops.fused_linear_cross_entropy(h2, w.detach(), labels, chunk_size=256, grad_hint=hint)
    (loss2 * weights).sum().div(div).backward()
    hf2 = h.detach().float().requires_grad_()
    lf2 = torch.nn.functional.cross_entropy(hf2 @ wf.detach().t(), labels, ignore_index=-100, reduction="none")
    (lf2 * weights).sum().div(div).backward()
    assert _rel_err(h2.grad, hf2.grad) < 2e-2


@cuda
def test_adamw_matches_torch():
    ops = _ops()
    torch.manual_seed(8)
    n = 10007
    p0 = torch.randn(n, device="cuda")
    p = p0.clone()
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    shadow = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.AdamW([ref], lr=1e-3, weight_decay=0.1, foreach=False)
    for step in range(1, 4):
        g = torch.randn(n, device="cuda")
        ops.adamw_step_(
            p, g, m, v, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.1, step=step, p_bf16=shadow
        )
        ref.grad = g.clone()
        opt.step()
    assert _rel_err(p, ref.detach()) < 1e-6
    assert torch.equal(shadow, p.bfloat16())


@cuda
def test_sumsq():
    ops = _ops()
    x = torch.randn(1_000_003, device="cuda")
    assert math.isclose(ops.sumsq(x).item(), x.double().pow(2).sum().item(), rel_tol=1e-4)
