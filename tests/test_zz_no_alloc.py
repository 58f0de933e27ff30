"""The allocation-free RMSNorm backward, called through its exported C symbol.

Callers that live inside another program's process (a C host application, a plugin in a
server that reserved all device memory) cannot call cudaMalloc or use PyTorch's allocator;
``rb_rmsnorm_bwd_noalloc`` serves them with a static device scratch array.  This test calls
the symbol with ctypes, exactly as such a caller would, and checks it against the regular
(allocating) entry point on two calls in a row.  The file is named so that pytest collects it
last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    from resihp_megatron_b200.ops import _build

    mod = _build.ext()  # loads (and if needed builds) the extension that exports the symbol
    lib = ctypes.CDLL(mod.__file__)
    fn = lib.rb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    cap = lib.rb_rmsnorm_bwd_noalloc_capacity
    cap.restype = ctypes.c_longlong
    cap.argtypes = []
    return fn, cap


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _rmsnorm_bwd_fp32(x, w, dy, dres, dw0, accumulate, eps=1e-5):
    """fp32 PyTorch oracle: autograd through ``y = x * rsqrt(mean(x^2) + eps) * w``."""
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * wf
    y.backward(dy.float())
    dx = xf.grad + (dres.float() if dres is not None else 0)
    dw = wf.grad + (dw0 if accumulate else 0)
    return dx, dw


@pytest.mark.parametrize("accumulate", [0, 1])
@pytest.mark.parametrize("with_dres", [False, True])
def test_noalloc_rmsnorm_bwd_matches_allocating_entry_point(accumulate, with_dres):
    from resihp_megatron_b200 import ops

    fn, cap = _entry()
    assert cap() == 512 * 1024
    T, H = 1000, 4096
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(7 + 2 * accumulate + int(with_dres))
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).bfloat16()
    _, rstd = ops.rmsnorm_fwd(x, w, 1e-5)
    for call in range(2):  # two calls in a row: the second sees the first call's scratch contents
        dy = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        dres = torch.randn(T, H, device="cuda", generator=g).bfloat16() if with_dres else None
        dw0 = torch.full((H,), 0.25, device="cuda")
        dw_ref = dw0.clone()
        dx_ref = ops.rmsnorm_bwd(x, w, rstd, dy, dw_ref, dres=dres, accumulate=bool(accumulate))
        dx = torch.empty_like(x)
        dw = torch.full((H,), -7.0 if not accumulate else 0.25, device="cuda")  # overwritten unless accumulating
        rc = fn(x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
                dres.data_ptr() if dres is not None else None, dx.data_ptr(), dw.data_ptr(), accumulate, T, H,
                stream)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: rb_rmsnorm_bwd_noalloc returned {rc}"
        # the same kernels as the allocating entry point: the same bits
        assert torch.equal(dx, dx_ref), call
        assert torch.equal(dw, dw_ref), call
        # and both agree with an fp32 PyTorch RMSNorm backward
        dx32, dw32 = _rmsnorm_bwd_fp32(x, w, dy, dres, dw0, accumulate)
        assert _rel(dx, dx32) < 1e-2, (call, _rel(dx, dx32))
        assert _rel(dw, dw32) < 1e-3, (call, _rel(dw, dw32))


def test_noalloc_rejects_oversized_calls():
    fn, cap = _entry()
    H = 8192
    T = (cap() // H + 1) * 32  # needs ceil(T/32) * H > capacity
    rc = fn(None, None, None, None, None, None, None, 1, T, H, torch.cuda.current_stream().cuda_stream)
    assert rc == -2
    assert fn(None, None, None, None, None, None, None, 1, 64, 12, 0) == -3
