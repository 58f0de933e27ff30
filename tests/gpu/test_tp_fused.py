"""Fused tensor-parallel GEMMs with emulated ranks on one GPU (each rank's kernel runs alone; the
kernels never wait on another launch): all-gather -> GEMM and GEMM -> reduce-scatter against an
fp32 reference of the same collective + GEMM."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,M,K,N", [(2, 512, 256, 512), (4, 1024, 512, 768), (8, 2048, 384, 256)])
def test_all_gather_gemm(world, M, K, N):
    from resihp_megatron_b200.ops.gemm import error_state
    from resihp_megatron_b200.parallel.tp_fused import TensorParallelComm

    ranks = TensorParallelComm.emulated_group(world, "cuda", max_rows=M, max_k=K, max_n=N)
    torch.manual_seed(0)
    rows = M // world
    xs = [torch.randn(rows, K, device="cuda").bfloat16() for _ in range(world)]
    ws = [torch.randn(N, K, device="cuda").bfloat16() for _ in range(world)]
    for r, t in enumerate(ranks):
        t.local_chunk(M, K).copy_(xs[r])
    torch.cuda.synchronize()
    x_all = torch.cat(xs).float()
    for r, t in enumerate(ranks):
        y = t.all_gather_gemm(M, ws[r])
        torch.cuda.synchronize()
        assert int(error_state()[0]) == 0
        ref = x_all @ ws[r].float().t()
        assert (y.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-2, r
        assert torch.equal(t.gather_buffer(M, K, buf=0), x_all.bfloat16()), "the gather buffer holds every chunk"
    ranks[0].close()


@pytest.mark.parametrize("world,M,K,N", [(2, 512, 256, 512), (4, 1024, 512, 768), (8, 2048, 384, 256)])
def test_gemm_reduce_scatter(world, M, K, N):
    from resihp_megatron_b200.parallel.tp_fused import TensorParallelComm

    ranks = TensorParallelComm.emulated_group(world, "cuda", max_rows=M, max_k=K, max_n=N)
    torch.manual_seed(1)
    xs = [torch.randn(M, K, device="cuda").bfloat16() for _ in range(world)]
    ws = [torch.randn(N, K, device="cuda").bfloat16() for _ in range(world)]
    for r, t in enumerate(ranks):
        t.scatter_partials(xs[r], ws[r])
    parts = [(xs[r].float() @ ws[r].float().t()).bfloat16().float() for r in range(world)]
    full = sum(parts)
    rows = M // world
    res = [torch.randn(rows, N, device="cuda").bfloat16() for _ in range(world)]
    outs = [t.reduce_received(M, N, residual=res[q]) for q, t in enumerate(ranks)]
    full = full + torch.cat(res).float()
    torch.cuda.synchronize()
    for q, y in enumerate(outs):
        ref = full[q * rows:(q + 1) * rows]
        assert (y.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 2e-2, q
    ranks[0].close()


@pytest.mark.parametrize("world", [2, 4])
def test_transposed_weight_variants(world):
    """The backward forms: all-gather -> GEMM and GEMM -> reduce-scatter with the weight read
    MN-major (``w_t``), as the input-gradient GEMMs of row- and column-parallel layers use it."""
    from resihp_megatron_b200.parallel.tp_fused import TensorParallelComm

    M, K, N = 512, 384, 256
    ranks = TensorParallelComm.emulated_group(world, "cuda", max_rows=M, max_k=max(K, N), max_n=max(K, N))
    torch.manual_seed(2)
    rows = M // world
    xs = [torch.randn(rows, K, device="cuda").bfloat16() for _ in range(world)]
    wts = [torch.randn(K, N, device="cuda").bfloat16() for _ in range(world)]  # stored [K, N]
    for r, t in enumerate(ranks):
        t.local_chunk(M, K).copy_(xs[r])
    x_all = torch.cat(xs).float()
    for r, t in enumerate(ranks):
        y = t.all_gather_gemm(M, wts[r], w_t=True, advance=False)
        ref = x_all @ wts[r].float()
        assert (y.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-2
    xf = [torch.randn(M, K, device="cuda").bfloat16() for _ in range(world)]
    for r, t in enumerate(ranks):
        t.scatter_partials(xf[r], wts[r], w_t=True)
    full = sum((xf[r].float() @ wts[r].float()).bfloat16().float() for r in range(world))
    for q, t in enumerate(ranks):
        y = t.reduce_received(M, N)
        ref = full[q * rows:(q + 1) * rows]
        assert (y.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 2e-2
    # plain gather
    for r, t in enumerate(ranks):
        g = t.all_gather(M, K, advance=False)
        assert torch.equal(g, x_all.bfloat16())
    ranks[0].close()


@pytest.mark.parametrize("world", [2, 4])
def test_fp8_all_gather_and_fp8_gemm_reduce_scatter(world):
    """Block-scaled fp8 under tensor parallelism: every rank quantises its rows (row-major scales)
    into the gather buffer and the fp8 gather moves rows and scales (bit-identical to quantising
    the gathered tensor); the fp8 GEMM's scatter epilogue feeds the rank-ordered reduction."""
    from resihp_megatron_b200.ops import fp8
    from resihp_megatron_b200.parallel.tp_fused import TensorParallelComm

    M, K, N = 1024, 512, 256
    ranks = TensorParallelComm.emulated_group(world, "cuda", max_rows=M, max_k=K, max_n=N)
    torch.manual_seed(2)
    rows = M // world
    xs = [torch.randn(rows, K, device="cuda").bfloat16() for _ in range(world)]
    for r, t in enumerate(ranks):
        q, s = t.fp8_local(M, K)
        local = fp8.Fp8Tensor(rows, K, fp8.E4M3, False, q.view(fp8.DTYPES[fp8.E4M3]), s, None, None, True)
        fp8.quantize(xs[r], fp8.E4M3, out=local)
    torch.cuda.synchronize()
    ref = fp8.quantize_reference(torch.cat(xs), fp8.E4M3, row_major=True)
    for t in ranks:
        q, s = t.all_gather_fp8(M, K, advance=False)
        torch.cuda.synchronize()
        assert torch.equal(q, ref.q_row.view(torch.uint8)) and torch.equal(s, ref.s_row)
    # row-parallel fp8 GEMM -> reduce-scatter through the scatter epilogue
    a = [fp8.quantize(torch.randn(M, K, device="cuda").bfloat16(), fp8.E4M3) for _ in range(world)]
    w = [fp8.quantize((torch.randn(N, K, device="cuda") * 0.05).bfloat16(), fp8.E4M3, two_d=True)
         for _ in range(world)]
    for r, t in enumerate(ranks):
        fp8.gemm(a[r].rowwise(), w[r].rowwise(), scatter=(t.heap.peer_ptrs(f"rs_recv{t._rs}"), r))
    parts = [fp8.gemm_reference(a[r].rowwise(), w[r].rowwise(), out_dtype=torch.bfloat16).float()
             for r in range(world)]
    full = sum(parts)
    outs = [t.reduce_received(M, N) for t in ranks]
    torch.cuda.synchronize()
    for q, y in enumerate(outs):
        want = full[q * rows:(q + 1) * rows]
        assert (y.float() - want).abs().max().item() <= 2e-2 * want.abs().max().item() + 1e-3, q
    ranks[0].close()
