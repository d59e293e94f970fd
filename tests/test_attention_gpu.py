"""Varlen flash attention (tcgen05) against a per-document fp32 oracle."""

import pytest
import torch

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _case(lens, Hq, Hkv, seed=0):
    torch.manual_seed(seed)
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device="cuda")
    q = torch.randn(T, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    return q, k, v, cu, max(lens)


CASES = [
    ([128], 2, 1),
    ([256], 4, 2),
    ([300, 212], 4, 4),
    ([1, 77, 129, 1000], 8, 2),
    ([256, 4096, 1333, 2507], 32, 8),
]


@cuda
@pytest.mark.parametrize("lens,Hq,Hkv", CASES)
@pytest.mark.parametrize("causal", [True, False])
def test_flash_fwd(lens, Hq, Hkv, causal):
    from mvp_engine.ops import _ext
    from mvp_engine.ops.attention import attention_reference

    q, k, v, cu, mx = _case(lens, Hq, Hkv)
    o, lse = _ext.ext().flash_attn_fwd(q, k, v, cu, 128**-0.5, causal, _ext.status_buffer().data_ptr())
    ref, ref_lse = attention_reference(q, k, v, cu, causal, 128**-0.5, return_lse=True)
    torch.cuda.synchronize()
    _ext.check_status()
    assert _rel(o, ref) < 1e-2, _rel(o, ref)
    assert torch.allclose(lse, ref_lse, atol=2e-2, rtol=1e-3)


@cuda
def test_flash_strided_v():
    """v as a strided view into a fused qkv buffer (the layout the model uses)."""
    from mvp_engine.ops.attention import attention_reference, flash_attn_varlen

    torch.manual_seed(1)
    T, Hq, Hkv = 700, 8, 2
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device="cuda").bfloat16()
    q = qkv[:, : Hq * 128].reshape(T, Hq, 128).contiguous()
    k = qkv[:, Hq * 128 : (Hq + Hkv) * 128].reshape(T, Hkv, 128).contiguous()
    v = qkv[:, (Hq + Hkv) * 128 :].view(T, Hkv, 128)
    cu = torch.tensor([0, 300, 700], dtype=torch.int32, device="cuda")
    o = flash_attn_varlen(q, k, v, cu, 400, causal=True)
    ref = attention_reference(q, k, v.contiguous(), cu, True)
    assert _rel(o, ref) < 1e-2


@cuda
@pytest.mark.parametrize("lens,Hq,Hkv", CASES[:4])
def test_flash_bwd(lens, Hq, Hkv):
    from mvp_engine.ops.attention import attention_reference, flash_attn_varlen

    q, k, v, cu, mx = _case(lens, Hq, Hkv, seed=3)
    q, k, v = (t.requires_grad_() for t in (q, k, v))
    o = flash_attn_varlen(q, k, v, cu, mx, causal=True)
    g = torch.randn_like(o)
    o.backward(g)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = attention_reference(qf, kf, vf, cu, True)
    ref.backward(g.float())
    assert _rel(o, ref) < 1e-2
    assert _rel(q.grad, qf.grad) < 2e-2
    assert _rel(k.grad, kf.grad) < 2e-2
    assert _rel(v.grad, vf.grad) < 2e-2


def _pair_case(lq, lk, Hq, Hkv, seed=0):
    """Query and key streams with their own document lengths (some empty on one side)."""
    torch.manual_seed(seed)
    cu_q = torch.tensor([0] + torch.tensor(lq).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    cu_k = torch.tensor([0] + torch.tensor(lk).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    q = torch.randn(sum(lq), Hq, 128, device="cuda").bfloat16()
    k = torch.randn(sum(lk), Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(sum(lk), Hkv, 128, device="cuda").bfloat16()
    return q, k, v, cu_q, cu_k


PAIR_CASES = [
    ([200, 0, 312], [100, 50, 362], False),
    ([64, 448], [0, 700], False),
    ([300, 212], [300, 212], True),
    ([256, 129], [512, 129], True),  # causal aligned to the document end
]


@cuda
@pytest.mark.parametrize("lq,lk,causal", PAIR_CASES)
def test_flash_pair_fwd_bwd(lq, lk, causal):
    """Separate key documents (the ring context-parallel building block) vs the fp32 oracle."""
    from mvp_engine.ops import _ext
    from mvp_engine.ops.attention import attention_pair_bwd_reference, attention_pair_reference

    q, k, v, cu_q, cu_k = _pair_case(lq, lk, 8, 2)
    ext = _ext.ext()
    st = _ext.status_buffer(q.device)
    o, lse = ext.flash_attn_fwd(q, k, v, cu_q, 128**-0.5, causal, st.data_ptr(), cu_seqlens_k=cu_k)
    ro, rl = attention_pair_reference(q, k, v, cu_q, cu_k, causal, 128**-0.5)
    torch.cuda.synchronize()
    _ext.check_status(q.device)
    assert _rel(o, ro) < 1e-2
    fin = torch.isfinite(rl)
    assert torch.equal(torch.isfinite(lse), fin)
    assert (lse[fin] - rl[fin]).abs().max().item() < 2e-2
    do = torch.randn_like(q)
    dq, dk, dv = ext.flash_attn_bwd(do, q, k, v, o, lse, cu_q, 128**-0.5, causal, st.data_ptr(), cu_seqlens_k=cu_k)
    rq, rk, rv = attention_pair_bwd_reference(do, q, k, v, o, lse, cu_q, cu_k, causal, 128**-0.5)
    torch.cuda.synchronize()
    _ext.check_status(q.device)
    for a, b in ((dq, rq), (dk, rk), (dv, rv)):
        assert _rel(a, b) < 2e-2
