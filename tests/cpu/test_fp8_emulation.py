"""Block-scaled fp8 emulation (the oracle of the fp8 kernels): power-of-two scale exponents
against a brute-force search, the operand addressing of every layout (rowwise / colwise,
1 x 128 / 128 x 128) against the tensor it came from, and the three GEMMs of a linear layer
against fp32 products."""

import math

import pytest
import torch

from resihp_megatron_b200.ops import fp8


@pytest.mark.parametrize("fmt", [fp8.E4M3, fp8.E5M2])
def test_scale_exponent_is_the_smallest_that_fits(fmt):
    fmax = 1.75 * 2.0 ** fp8.MAX_EXP[fmt]
    vals = [1e-45, 1e-40, 1.1754944e-38, 1e-30, 0.3, 0.5, 1.0, 1.75, 1.7500001, fmax, fmax * 1.0000001, 2.0 ** 20,
            3e38]
    vals += torch.logspace(-20, 20, 97).tolist()
    e = fp8.scale_exponent(torch.tensor(vals), fmt)
    for v, got in zip(vals, e.tolist()):
        v32 = torch.tensor(v, dtype=torch.float32).item()
        want = min(k for k in range(-300, 300) if v32 * 2.0 ** (-k) <= fmax)
        assert got == max(-126, min(126, want)), (v32, got, want)
    special = fp8.scale_exponent(torch.tensor([0.0, float("inf"), float("nan")]), fmt)
    assert special.tolist() == [0, 0, 0]


def _tensor(R=256, C=384, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(R, C, generator=g) * torch.logspace(-3, 3, C)[None, :]
    x[3, 5] = 3000.0
    return x.bfloat16()


@pytest.mark.parametrize("two_d", [False, True])
@pytest.mark.parametrize("fmt", [fp8.E4M3, fp8.E5M2])
def test_operand_views_dequantize_to_the_tensor(fmt, two_d):
    x = _tensor()
    amax = torch.zeros(1)
    t = fp8.quantize_reference(x, fmt, two_d=two_d, rowwise=True, colwise=True, amax=amax)
    assert amax.item() == x.float().abs().max().item()
    mbits = 3 if fmt == fp8.E4M3 else 2
    for op, ref in ((t.rowwise(), x.float()), (t.colwise(), x.float().t())):
        assert op.data.dtype == fp8.DTYPES[fmt] and op.data.is_contiguous()
        s = op.scale_matrix()
        assert torch.equal(s, fp8.pow2(torch.log2(s).round().to(torch.int64)))  # powers of two
        q = op.data.float()
        assert q.abs().max() <= 1.75 * 2.0 ** fp8.MAX_EXP[fmt]
        d = op.dequantize()
        # within half a unit in the last place of the block's largest magnitude, relative to it
        bs = s.repeat_interleave(fp8.BLOCK, 1)
        assert ((d - ref).abs() <= bs * 2.0 ** (fp8.MAX_EXP[fmt] - mbits)).all()
        # normal-range values keep mbits of precision
        big = ref.abs() >= bs * 2.0 ** (-6 if fmt == fp8.E4M3 else -14)
        assert ((d - ref).abs()[big] <= ref.abs()[big] * 2.0 ** -(mbits + 1) * 1.0001).all()


def test_two_d_scales_are_shared_by_both_layouts():
    x = _tensor(384, 256, 1)
    t = fp8.quantize_reference(x, fp8.E4M3, two_d=True, rowwise=True, colwise=True)
    grid = t.rowwise().scale_matrix()[::128]  # [R/128, C/128]: one scale per 128 x 128 tile
    assert torch.equal(grid.repeat_interleave(128, 0), t.rowwise().scale_matrix())
    assert torch.equal(grid.t().repeat_interleave(128, 0), t.colwise().scale_matrix())
    assert torch.equal(t.q_col.float(), t.q_row.float().t())


def test_linear_layer_gemms_match_fp32():
    torch.manual_seed(0)
    T, H, F = 256, 384, 512
    x = torch.randn(T, H).bfloat16()
    w = (torch.randn(F, H) * 0.05).bfloat16()
    dy = (torch.randn(T, F) * 1e-3).bfloat16()
    xq = fp8.quantize_reference(x, fp8.E4M3, rowwise=True, colwise=True)
    wq = fp8.quantize_reference(w, fp8.E4M3, two_d=True, rowwise=True, colwise=True)
    dyq = fp8.quantize_reference(dy, fp8.E5M2, rowwise=True, colwise=True)

    def rel(a, b):
        return ((a.float() - b).norm() / b.norm()).item()

    y = fp8.gemm_reference(xq.rowwise(), wq.rowwise(), out_dtype=torch.float32)
    assert rel(y, x.float() @ w.float().t()) < 0.05
    dx = fp8.gemm_reference(dyq.rowwise(), wq.colwise(), out_dtype=torch.float32)
    assert rel(dx, dy.float() @ w.float()) < 0.1
    g = torch.ones(F, H)
    fp8.gemm_reference(dyq.colwise(), xq.colwise(), out=g, accumulate=True)
    assert rel(g - 1.0, dy.float().t() @ x.float()) < 0.1
    # exactly the dequantised product
    ref = xq.rowwise().dequantize() @ wq.rowwise().dequantize().t()
    assert torch.allclose(y, ref, rtol=1e-5, atol=1e-5)


def test_rejects_unaligned_shapes():
    with pytest.raises(ValueError):
        fp8.quantize_reference(torch.zeros(100, 128).bfloat16(), colwise=True)
    with pytest.raises(ValueError):
        fp8.quantize_reference(torch.zeros(128, 100).bfloat16())
    part = fp8.quantize_reference(torch.ones(100, 128).bfloat16(), row_major=True)  # rowwise-only: any rows
    assert part.rowwise().dequantize().eq(1).all() and part.s_row.shape == (100, 1)
    with pytest.raises(ValueError):
        fp8.Fp8Tensor.empty(128, 200)
    assert math.isclose(1.75 * 2 ** fp8.MAX_EXP[fp8.E4M3], 448.0)
    assert math.isclose(1.75 * 2 ** fp8.MAX_EXP[fp8.E5M2], 57344.0)


def test_gemm_validates_shapes_and_scales_before_any_native_call(monkeypatch):
    """Every operand rule of the fp8 GEMM is checked in Python: a bad shape or a scale vector too
    short for its addressing never reaches the extension."""

    def _no_native_call():
        raise AssertionError("a bad operand reached the extension")

    monkeypatch.setattr(fp8, "ext", _no_native_call)
    q = fp8.quantize_reference(torch.ones(128, 256).bfloat16())
    good = q.rowwise()
    short_k = fp8.Fp8Operand(good.data[:, :64].contiguous(), good.scale, good.kb_stride, 1, 0, fp8.E4M3)
    with pytest.raises(fp8.Fp8ShapeError, match="multiples of 128"):
        fp8.gemm(short_k, short_k)
    few_scales = fp8.Fp8Operand(good.data, good.scale[:1].contiguous(), good.kb_stride, 1, 0, fp8.E4M3)
    with pytest.raises(fp8.Fp8ShapeError, match="cannot cover"):
        fp8.gemm(few_scales, good)
    bad_shift = fp8.Fp8Operand(good.data, good.scale, good.kb_stride, 1, 3, fp8.E4M3)
    with pytest.raises(fp8.Fp8ShapeError, match="addressing"):
        fp8.gemm(good, bad_shift)
    other_k = fp8.quantize_reference(torch.ones(128, 384).bfloat16()).rowwise()
    with pytest.raises(fp8.Fp8ShapeError, match="contraction"):
        fp8.gemm(good, other_k)
    # the error is both a ValueError and a RuntimeError (callers catching either keep working)
    assert issubclass(fp8.Fp8ShapeError, ValueError) and issubclass(fp8.Fp8ShapeError, RuntimeError)


def test_kernel_choice_by_product_size():
    """``variant=0`` sends products under ``SMALL_FLOPS`` to the register-promotion kernel (one
    launch) when B's scales allow it, everything else to the block-scaled MMA (two scale-packing
    launches + the GEMM); the launch count reported for a call follows the same rule."""
    import torch

    def op(rows, K, shift, row_stride=1, kb_stride=None):
        nkb = K // 128
        scale = torch.ones(max(1, (rows >> shift)) * nkb + 16)
        kb_stride = (rows >> shift) if kb_stride is None else kb_stride
        return fp8.Fp8Operand(torch.zeros(rows, K, dtype=torch.uint8), scale, kb_stride, row_stride, shift, fp8.E4M3)

    small_a, small_b = op(4096, 2048, 0), op(1024, 2048, 7)     # 1.7e10 FLOPs
    big_a, big_b = op(4096, 2048, 0), op(4096, 2048, 7)         # 6.9e10 FLOPs
    assert fp8._promotes(small_a, small_b, 0) and fp8._launches(small_a, small_b, 0) == 1
    assert not fp8._promotes(big_a, big_b, 0) and fp8._launches(big_a, big_b, 0) == 3
    assert not fp8._promotes(small_a, small_b, 2) and fp8._promotes(big_a, big_b, 1)
    # per-column B scales the promotion kernel cannot read (K-block stride not a multiple of 4)
    odd = op(1024, 2048, 0, kb_stride=1026)
    assert not fp8._promotes(small_a, odd, 0)
