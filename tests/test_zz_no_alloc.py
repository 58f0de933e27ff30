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


def test_noalloc_rmsnorm_bwd_matches_allocating_entry_point():
    from resihp_megatron_b200 import ops

    fn, cap = _entry()
    assert cap() == 512 * 1024
    T, H = 1000, 4096
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).bfloat16()
    _, rstd = ops.rmsnorm_fwd(x, w, 1e-5)
    for call in range(2):  # two calls in a row: the second sees the first call's scratch contents
        dy = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        dres = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        dw_ref = torch.full((H,), 0.25, device="cuda")
        dx_ref = ops.rmsnorm_bwd(x, w, rstd, dy, dw_ref, dres=dres, accumulate=True)
        dx = torch.empty_like(x)
        dw = torch.full((H,), 0.25, device="cuda")
        rc = fn(x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dy.data_ptr(), dres.data_ptr(), dx.data_ptr(),
                dw.data_ptr(), 1, T, H, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: rb_rmsnorm_bwd_noalloc returned {rc}"
        assert _rel(dx, dx_ref) < 1e-2, call
        assert _rel(dw, dw_ref) < 1e-3, call


def test_noalloc_rejects_oversized_calls():
    fn, cap = _entry()
    H = 8192
    T = (cap() // H + 1) * 32  # needs ceil(T/32) * H > capacity
    rc = fn(None, None, None, None, None, None, None, 1, T, H, torch.cuda.current_stream().cuda_stream)
    assert rc == -2
    assert fn(None, None, None, None, None, None, None, 1, 64, 12, 0) == -3
