"""Numerics of the tcgen05 GEMM against a plain PyTorch fp32 reference of the same op."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, a_t, b_t):
    A = (a.t() if a_t else a).float()
    B = (b.t() if b_t else b).float()
    return A @ B.t()


def _mk(M, N, K, a_t, b_t, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn((K, M) if a_t else (M, K), device="cuda", generator=g).bfloat16()
    b = torch.randn((K, N) if b_t else (N, K), device="cuda", generator=g).bfloat16()
    return a, b


SHAPES = [(128, 128, 64), (256, 512, 256), (384, 256, 1024), (1000, 296, 200), (136, 520, 72)]


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bf16_out(M, N, K, a_t, b_t):
    from resihp_megatron_b200.ops.gemm import gemm, error_state

    a, b = _mk(M, N, K, a_t, b_t)
    out = gemm(a, b, a_t=a_t, b_t=b_t)
    ref = _ref(a, b, a_t, b_t)
    torch.cuda.synchronize()
    assert int(error_state()[0]) == 0
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-2 * scale + 1e-2, (err, scale)


@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (1000, 296, 200)])
def test_gemm_fp32_accumulate(M, N, K):
    from resihp_megatron_b200.ops.gemm import gemm

    a, b = _mk(M, N, K, True, True, seed=1)
    base = torch.randn(M, N, device="cuda")
    out = base.clone()
    gemm(a, b, a_t=True, b_t=True, out=out, accumulate=True)
    ref = base + _ref(a, b, True, True)
    torch.cuda.synchronize()
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-3), (out - ref).abs().max().item()
    out2 = gemm(a, b, a_t=True, b_t=True, out_dtype=torch.float32, alpha=0.5)
    assert torch.allclose(out2, 0.5 * _ref(a, b, True, True), rtol=1e-4, atol=1e-3)


def test_gemm_residual():
    from resihp_megatron_b200.ops.gemm import gemm

    a, b = _mk(512, 768, 384, False, False, seed=2)
    r = torch.randn(512, 768, device="cuda").bfloat16()
    out = gemm(a, b, residual=r)
    ref = _ref(a, b, False, False) + r.float()
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 2e-2


def test_gemm_large_square():
    from resihp_megatron_b200.ops.gemm import gemm

    a, b = _mk(4096, 4096, 4096, False, False, seed=3)
    out = gemm(a, b)
    ref = _ref(a, b, False, False)
    torch.cuda.synchronize()
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err


PAIR_SHAPES = [(256, 256, 64), (640, 384, 320), (1000, 520, 200), (512, 1024, 1024)]


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
def test_gemm_cta_pair_variant(M, N, K, a_t, b_t):
    """The 2-CTA (cta_group::2) kernel against fp32 and against the single-CTA kernel, with every
    epilogue (bf16, fp32, fp32 accumulate, bf16 + residual)."""
    from resihp_megatron_b200.ops.gemm import error_state, gemm

    a, b = _mk(M, N, K, a_t, b_t, seed=7)
    ref = _ref(a, b, a_t, b_t)
    scale = ref.abs().max().item()
    pair = gemm(a, b, a_t=a_t, b_t=b_t, variant=2)
    single = gemm(a, b, a_t=a_t, b_t=b_t, variant=1)
    f32 = gemm(a, b, a_t=a_t, b_t=b_t, out_dtype=torch.float32, variant=2)
    base = torch.randn(M, N, device="cuda")
    acc = base.clone()
    gemm(a, b, a_t=a_t, b_t=b_t, out=acc, accumulate=True, variant=2)
    r = torch.randn(M, N, device="cuda").bfloat16()
    res = gemm(a, b, a_t=a_t, b_t=b_t, residual=r, variant=2)
    torch.cuda.synchronize()
    assert int(error_state()[0]) == 0
    assert (pair.float() - ref).abs().max().item() <= 1e-2 * scale + 1e-2
    assert torch.equal(pair, single), "same math and summation order as the single-CTA kernel"
    assert torch.allclose(f32, ref, rtol=1e-4, atol=1e-3)
    assert torch.allclose(acc, base + ref, rtol=1e-4, atol=1e-3)
    assert (res.float() - (ref + r.float())).abs().max().item() <= 1e-2 * scale + 2e-2


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(512, 1024, 1024), (1000, 520, 1000), (256, 256, 192)])
def test_gemm_split_k_variant(M, N, K, a_t, b_t):
    """Split-K of the CTA-pair kernel (variant 3: two k shares per tile, partials reduced by the
    last-arriving unit) against fp32 with every epilogue, against the unsplit pair kernel, and
    bitwise equal from run to run (the reduction order does not depend on arrival order)."""
    from resihp_megatron_b200.ops.gemm import error_state, gemm

    a, b = _mk(M, N, K, a_t, b_t, seed=11)
    ref = _ref(a, b, a_t, b_t)
    scale = ref.abs().max().item()
    split = gemm(a, b, a_t=a_t, b_t=b_t, variant=3)
    again = gemm(a, b, a_t=a_t, b_t=b_t, variant=3)
    whole = gemm(a, b, a_t=a_t, b_t=b_t, variant=2)
    f32 = gemm(a, b, a_t=a_t, b_t=b_t, out_dtype=torch.float32, variant=3)
    base = torch.randn(M, N, device="cuda")
    acc = base.clone()
    gemm(a, b, a_t=a_t, b_t=b_t, out=acc, accumulate=True, variant=3)
    r = torch.randn(M, N, device="cuda").bfloat16()
    res = gemm(a, b, a_t=a_t, b_t=b_t, residual=r, variant=3, alpha=0.5)
    torch.cuda.synchronize()
    assert int(error_state()[0]) == 0
    assert (split.float() - ref).abs().max().item() <= 1e-2 * scale + 1e-2
    assert torch.equal(split, again)
    assert (split.float() - whole.float()).abs().max().item() <= 1e-2 * scale + 1e-2
    assert torch.allclose(f32, ref, rtol=1e-4, atol=1e-3)
    assert torch.allclose(acc, base + ref, rtol=1e-4, atol=1e-3)
    assert (res.float() - (0.5 * ref + r.float())).abs().max().item() <= 1e-2 * scale + 2e-2


def test_gemm_auto_split_on_a_partial_wave_shape():
    """M = N = 4096 is 256 pair tiles (3.46 waves on 74 pairs); at K = 8192 the default variant
    splits the partial last wave's tiles: within bf16 rounding of fp32 and deterministic."""
    from resihp_megatron_b200.ops.gemm import error_state, gemm

    a, b = _mk(4096, 4096, 8192, False, True, seed=12)
    out = gemm(a, b, b_t=True)
    out2 = gemm(a, b, b_t=True)
    ref = _ref(a, b, False, True)
    torch.cuda.synchronize()
    assert int(error_state()[0]) == 0
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    assert torch.equal(out, out2)


@pytest.mark.parametrize("variant", [4, 5])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(512, 1024, 1024), (1000, 520, 1000)])
def test_gemm_pair_ring_and_tile_variants_match(M, N, K, a_t, b_t, variant):
    """The CTA-pair kernel with a 7-stage operand ring (variant 4) or 256 x 128 tiles (variant 5)
    computes the same sums in the same k order as the default 6-stage 256 x 256 one: bitwise
    equal, every operand layout, bf16 and fp32-accumulate epilogues."""
    from resihp_megatron_b200.ops.gemm import error_state, gemm

    a, b = _mk(M, N, K, a_t, b_t, seed=13)
    assert torch.equal(gemm(a, b, a_t=a_t, b_t=b_t, variant=variant), gemm(a, b, a_t=a_t, b_t=b_t, variant=2))
    base = torch.randn(M, N, device="cuda")
    acc6, acc7 = base.clone(), base.clone()
    gemm(a, b, a_t=a_t, b_t=b_t, out=acc6, accumulate=True, variant=2)
    gemm(a, b, a_t=a_t, b_t=b_t, out=acc7, accumulate=True, variant=variant)
    torch.cuda.synchronize()
    assert int(error_state()[0]) == 0
    assert torch.equal(acc6, acc7)


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096), (2048, 3072, 4096)])
def test_gemm_tail_split_variant(M, N, K):
    """Variant 6 splits only the tiles of the partial last wave (2 shares for 256 tiles on 74 SM
    pairs, 3 for 96 tiles): within bf16 rounding of fp32 and of the unsplit kernel, fp32
    accumulation exact to fp32 tolerance, and bitwise equal run to run."""
    from resihp_megatron_b200.ops.gemm import error_state, gemm

    a, b = _mk(M, N, K, False, True, seed=14)
    ref = _ref(a, b, False, True)
    scale = ref.abs().max().item()
    out = gemm(a, b, b_t=True, variant=6)
    again = gemm(a, b, b_t=True, variant=6)
    whole = gemm(a, b, b_t=True, variant=2)
    base = torch.randn(M, N, device="cuda")
    acc = base.clone()
    gemm(a, b, b_t=True, out=acc, accumulate=True, variant=6)
    torch.cuda.synchronize()
    assert int(error_state()[0]) == 0
    assert (out.float() - ref).abs().max().item() <= 1e-2 * scale
    assert (out.float() - whole.float()).abs().max().item() <= 1e-2 * scale
    assert torch.equal(out, again)
    assert torch.allclose(acc, base + ref, rtol=1e-4, atol=1e-3)
