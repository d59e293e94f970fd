"""The allocation-free RMSNorm backward entry point, called through its exported C symbol.

Callers that cannot allocate device memory while they run (pre-planned
executors, stream capture, real-time threads) use ``mvp_rmsnorm_bwd_noalloc``;
this checks it against the regular ``rmsnorm_bwd`` entry point on two calls in
a row (the second call reuses the shared scratch array left by the first) and
that oversized inputs are refused.  The file is named so pytest collects it
last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _entry():
    import mvp_engine._C as ext_mod

    fn = ctypes.CDLL(ext_mod.__file__).mvp_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _case(rows, hidden):
    from mvp_engine.ops import _ext

    ext = _ext.ext()
    torch.manual_seed(rows * 7 + hidden)
    x = torch.randn(rows, hidden, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(hidden, device="cuda")).bfloat16()
    dy = torch.randn(rows, hidden, device="cuda").bfloat16()
    _, rstd = ext.rmsnorm_fwd(x, None, w, 1e-6)
    ref_dx, ref_dw = ext.rmsnorm_bwd(dy, x, rstd, w, None, True)
    return x, w, dy, rstd, ref_dx, ref_dw


def _call_and_check(fn, rows, hidden, case):
    x, w, dy, rstd, ref_dx, ref_dw = case
    dx = torch.full_like(x, float("nan"))
    dw = torch.full((hidden,), float("nan"), device="cuda")
    rc = fn(dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), w.data_ptr(), dx.data_ptr(), dw.data_ptr(),
            rows, hidden, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert _rel(dx, ref_dx) < 1e-2
    assert _rel(dw, ref_dw) < 1e-4


@cuda
@pytest.mark.parametrize("rows,hidden", [(1000, 4096), (77, 1152), (5000, 256), (1, 4096), (5, 1152)])
def test_noalloc_rmsnorm_bwd_matches_regular_entry_point(rows, hidden):
    fn = _entry()
    case = _case(rows, hidden)
    for _ in range(2):  # the second call finds the first call's partial sums in the shared scratch
        _call_and_check(fn, rows, hidden, case)


@cuda
def test_noalloc_large_call_then_small_call():
    """A small call after a large one uses fewer scratch slots; the large call's leftovers must not leak in."""
    fn = _entry()
    _call_and_check(fn, 6000, 2048, _case(6000, 2048))
    _call_and_check(fn, 3, 2048, _case(3, 2048))
    _call_and_check(fn, 40, 2048, _case(40, 2048))


@cuda
def test_noalloc_rejects_oversized_hidden():
    fn = _entry()
    x = torch.zeros(4, 32768, device="cuda", dtype=torch.bfloat16)
    r = torch.ones(4, device="cuda")
    out = torch.zeros(32768, device="cuda")
    rc = fn(x.data_ptr(), x.data_ptr(), r.data_ptr(), x.data_ptr(), x.data_ptr(), out.data_ptr(), 4, 32768,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
