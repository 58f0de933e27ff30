"""Block-scaled fp8 kernels against their PyTorch emulation: the quantiser bit for bit (bytes,
scales, amax), the tcgen05 GEMM (all three scale layouts of a linear layer, every epilogue)
against the fp32 sum of the same block products, and GELU against PyTorch."""

import pytest
import torch

from resihp_megatron_b200.ops import fp8

pytestmark = pytest.mark.gpu


def _x(R, C, seed=0, spread=3.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(R, C, device="cuda", generator=g) * torch.logspace(-spread, spread, C, device="cuda")[None, :]
    return x.bfloat16()


@pytest.mark.parametrize("two_d", [False, True])
@pytest.mark.parametrize("fmt", [fp8.E4M3, fp8.E5M2])
def test_quantize_matches_emulation_bitwise(fmt, two_d):
    x = _x(384, 640, seed=fmt)
    x[7, 9] = 0.0
    x[128:256, 256:384] = 0.0  # an all-zero block / tile
    amax = torch.zeros(1, device="cuda")
    got = fp8.quantize(x, fmt, two_d=two_d, rowwise=True, colwise=True, amax=amax)
    ref_amax = torch.zeros(1, device="cuda")
    ref = fp8.quantize_reference(x, fmt, two_d=two_d, rowwise=True, colwise=True, amax=ref_amax)
    torch.cuda.synchronize()
    assert torch.equal(got.q_row.view(torch.uint8), ref.q_row.view(torch.uint8))
    assert torch.equal(got.q_col.view(torch.uint8), ref.q_col.view(torch.uint8))
    assert torch.equal(got.s_row, ref.s_row)
    if not two_d:
        assert torch.equal(got.s_col, ref.s_col)
    assert amax.item() == ref_amax.item() == x.float().abs().max().item()


def test_quantize_strided_input_and_running_amax():
    base = _x(256, 768, seed=3)
    x = base[:, 128:640]  # row stride 768
    amax = torch.full((1,), 1e6, device="cuda")
    got = fp8.quantize(x, fp8.E4M3, rowwise=True, amax=amax)
    ref = fp8.quantize_reference(x.contiguous(), fp8.E4M3, rowwise=True)
    assert torch.equal(got.q_row.view(torch.uint8), ref.q_row.view(torch.uint8))
    assert amax.item() == 1e6  # a running max keeps the larger value


def _check(out, ref, tol):
    err = (out.float() - ref.float()).abs().max().item()
    assert err <= tol * ref.float().abs().max().item() + 1e-30, err


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (1024, 1024, 2048), (256, 128, 128), (4096, 1280, 256)])
def test_gemm_forward_dgrad_wgrad(M, N, K, variant):
    """Variants 2 and 3 apply the scales in the tensor core (block-scaled MMA; single CTAs and CTA
    pairs), 1 in registers per K-block, 0 picks by size; all against the PyTorch emulation of the
    same block-scaled product.  The forward of 4096 x 1280 runs 160 tiles with a partly empty last column of tiles."""
    x = _x(M, K, seed=1, spread=1.0)
    w = (_x(N, K, seed=2, spread=0.5).float() * 0.05).bfloat16()
    dy = (_x(M, N, seed=4, spread=1.0).float() * 1e-3).bfloat16()
    xq = fp8.quantize(x, fp8.E4M3, rowwise=True, colwise=True)
    wq = fp8.quantize(w, fp8.E4M3, two_d=True, rowwise=True, colwise=True)
    dyq = fp8.quantize(dy, fp8.E5M2, rowwise=True, colwise=True)
    # forward: per-row A scales, 128 x 128 B scales
    y = fp8.gemm(xq.rowwise(), wq.rowwise(), out_dtype=torch.float32, variant=variant)
    _check(y, fp8.gemm_reference(xq.rowwise(), wq.rowwise(), out_dtype=torch.float32), 1e-5)
    yb = fp8.gemm(xq.rowwise(), wq.rowwise(), variant=variant)
    _check(yb, fp8.gemm_reference(xq.rowwise(), wq.rowwise(), out_dtype=torch.float32), 8e-3)
    # dgrad: E5M2 x E4M3, transposed 2-D weight scales
    dx = fp8.gemm(dyq.rowwise(), wq.colwise(), out_dtype=torch.float32, variant=variant)
    _check(dx, fp8.gemm_reference(dyq.rowwise(), wq.colwise(), out_dtype=torch.float32), 1e-5)
    # wgrad: per-column B scales, fp32 accumulate with alpha
    g0 = torch.randn(N, K, device="cuda")
    g = g0.clone()
    # the CTA-pair kernel needs the A rows (here N) in multiples of 256
    fp8.gemm(dyq.colwise(), xq.colwise(), out=g, accumulate=True, alpha=0.5,
             variant=variant if variant != 3 or N % 256 == 0 else 0)
    ref = g0.clone()
    fp8.gemm_reference(dyq.colwise(), xq.colwise(), out=ref, accumulate=True, alpha=0.5)
    _check(g - g0, ref - g0, 1e-5)
    # and the whole thing tracks the bf16 product
    full = (x.float() @ w.float().t())
    assert ((y - full).norm() / full.norm()).item() < 0.05


def test_gemm_rejects_unaligned(monkeypatch):
    a = fp8.quantize(_x(128, 128), fp8.E4M3)
    torch.cuda.synchronize()
    bad = fp8.Fp8Operand(a.q_row[:, :64].contiguous(), a.s_row, 128, 1, 0, fp8.E4M3)

    def _no_native_call():
        raise AssertionError("a bad shape reached the extension")

    # the shape error is raised in Python, before the extension is touched
    monkeypatch.setattr(fp8, "ext", _no_native_call)
    with pytest.raises(fp8.Fp8ShapeError, match="multiples of 128"):
        fp8.gemm(bad, bad)
    with pytest.raises(fp8.Fp8ShapeError, match="contraction"):
        fp8.gemm(a.rowwise(), fp8.Fp8Operand(torch.zeros(128, 256, dtype=torch.uint8, device="cuda"),
                                             torch.ones(256, device="cuda"), 128, 1, 0, fp8.E4M3))


def test_gelu_fwd_bwd():
    from resihp_megatron_b200 import ops

    h = (torch.randn(300, 1024, device="cuda") * 3).bfloat16()
    da = torch.randn(300, 1024, device="cuda").bfloat16()
    a = ops.gelu_fwd(h)
    hf = h.float().requires_grad_(True)
    ref = torch.nn.functional.gelu(hf, approximate="tanh")
    assert ((a.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2
    ref.backward(da.float())
    dh = ops.gelu_bwd(h, da)
    assert ((dh.float() - hf.grad).abs().max() / hf.grad.abs().max()).item() < 1e-2
    h2 = h.clone()
    ops.gelu_bwd(h2, da, out=h2)  # in place
    assert torch.equal(h2, dh)


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
def test_gemm_residual_and_scatter_epilogues(variant):
    M, N, K, world = 512, 256, 384, 4
    x = _x(M, K, seed=5, spread=1.0)
    w = (_x(N, K, seed=6, spread=0.5).float() * 0.05).bfloat16()
    res = _x(M, N, seed=7, spread=0.0)
    xq = fp8.quantize(x, fp8.E4M3)
    wq = fp8.quantize(w, fp8.E4M3, two_d=True)
    ref = fp8.gemm_reference(xq.rowwise(), wq.rowwise(), out_dtype=torch.float32)
    y = fp8.gemm(xq.rowwise(), wq.rowwise(), residual=res, variant=variant)
    _check(y, ref + res.float(), 8e-3)
    # scatter: rows of rank q's share land in slot 1 of buffer q ([world][M / world][N])
    rows = M // world
    bufs = [torch.zeros(world, rows, N, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    fp8.gemm(xq.rowwise(), wq.rowwise(), scatter=([b.data_ptr() for b in bufs], 1), variant=variant)
    full = fp8.gemm(xq.rowwise(), wq.rowwise(), variant=variant)
    for q in range(world):
        assert torch.equal(bufs[q][1], full[q * rows:(q + 1) * rows])
        assert bufs[q][0].abs().sum().item() == 0 and bufs[q][2:].abs().sum().item() == 0


@pytest.mark.parametrize("row_major", [False, True])
def test_rmsnorm_quantize_equals_norm_then_quantize(row_major):
    """The fused RMSNorm -> fp8 kernel writes the same bytes, scales, rstd and amax as
    ``rmsnorm_fwd`` followed by ``quantize`` (partial last row tile too)."""
    from resihp_megatron_b200 import ops

    T, H = 300, 2048
    x = _x(T, H, seed=9, spread=1.0)
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    y, rstd = ops.rmsnorm_fwd(x, w, 1e-5)
    a0 = torch.zeros(1, device="cuda")
    ref = fp8.quantize(y, fp8.E4M3, amax=a0, row_major=row_major)
    out = fp8.Fp8Tensor.empty(T, H, fp8.E4M3, device="cuda", row_major=row_major)
    r2 = torch.empty(T, device="cuda")
    a1 = torch.zeros(1, device="cuda")
    fp8.rmsnorm_quantize(x, w, 1e-5, fp8.E4M3, out=out, rstd=r2, amax=a1)
    torch.cuda.synchronize()
    assert torch.equal(out.q_row.view(torch.uint8), ref.q_row.view(torch.uint8))
    assert torch.equal(out.s_row, ref.s_row) and torch.equal(r2, rstd) and a0.item() == a1.item()


@pytest.mark.parametrize("gated", [False, True])
def test_act_quantize_equals_activation_then_quantize(gated):
    """GELU / SwiGLU written straight as fp8: same bytes, scales and amax as the bf16 activation
    kernel followed by ``quantize``."""
    from resihp_megatron_b200 import ops

    T, F = 257, 1024
    gu = _x(T, 2 * F if gated else F, seed=11, spread=0.5)
    y = ops.swiglu_fwd(gu) if gated else ops.gelu_fwd(gu)
    a0, a1 = torch.zeros(1, device="cuda"), torch.zeros(1, device="cuda")
    ref = fp8.quantize(y, fp8.E4M3, amax=a0)
    out = fp8.Fp8Tensor.empty(T, F, fp8.E4M3, device="cuda")
    fp8.act_quantize(gu, gated, fp8.E4M3, out=out, amax=a1)
    torch.cuda.synchronize()
    assert torch.equal(out.q_row.view(torch.uint8), ref.q_row.view(torch.uint8))
    assert torch.equal(out.s_row, ref.s_row) and a0.item() == a1.item()


@pytest.mark.parametrize("act", ["gelu", "swiglu"])
def test_quantize_of_the_activation_equals_activation_then_quantize(act):
    """The quantiser's activation option (the fp8 wgrad input of fc2, along tokens): same bytes and
    scales as the bf16 activation kernel followed by ``quantize``."""
    from resihp_megatron_b200 import ops

    T, F = 384, 1024
    gu = _x(T, 2 * F if act == "swiglu" else F, seed=12, spread=0.5)
    y = ops.swiglu_fwd(gu) if act == "swiglu" else ops.gelu_fwd(gu)
    ref = fp8.quantize(y, fp8.E4M3, rowwise=True, colwise=True)
    got = fp8.quantize(gu, fp8.E4M3, rowwise=True, colwise=True, act=act)
    torch.cuda.synchronize()
    assert torch.equal(got.q_row.view(torch.uint8), ref.q_row.view(torch.uint8))
    assert torch.equal(got.q_col.view(torch.uint8), ref.q_col.view(torch.uint8))
    assert torch.equal(got.s_row, ref.s_row) and torch.equal(got.s_col, ref.s_col)


def test_gemm_tensor_core_scaling_tracks_register_promotion_with_wide_scale_spread():
    """Rows of A and B whose magnitudes span many binades, so that every 1 x 128 row scale and
    every 128 x 128 weight scale differs: the tensor-core scaled products (per-row E8M0 words in
    TMEM; CTA pair and single CTA) and the register-promoted one all track the emulation to fp32
    summation order -- a scale placed on the wrong row, row group or CTA would not."""
    M, N, K = 512, 768, 1024
    g = torch.Generator(device="cuda").manual_seed(11)
    rs = torch.exp2(torch.randint(-12, 12, (M, 1), device="cuda", generator=g).float())
    cs = torch.exp2(torch.randint(-12, 12, (N, 1), device="cuda", generator=g).float())
    x = (torch.randn(M, K, device="cuda", generator=g) * rs).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * cs).bfloat16()
    xq = fp8.quantize(x, fp8.E4M3, rowwise=True)
    wq = fp8.quantize(w, fp8.E4M3, two_d=True, rowwise=True)
    wv = fp8.quantize(w, fp8.E4M3, rowwise=True)  # per-row B scales as well
    for b in (wq.rowwise(), wv.rowwise()):
        ref = fp8.gemm_reference(xq.rowwise(), b, out_dtype=torch.float32)
        # relative to each row's own magnitude: small rows must be right too
        scale = ref.abs().amax(dim=1, keepdim=True) + 1e-30
        for v in (3, 2, 1):  # CTA pair, single CTA, register promotion
            y = fp8.gemm(xq.rowwise(), b, out_dtype=torch.float32, variant=v)
            assert ((y - ref).abs() / scale).max().item() < 1e-5, v
