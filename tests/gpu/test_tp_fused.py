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
        assert torch.equal(t.gather_buffer(M, K), x_all.bfloat16()), "the gather buffer holds every chunk"
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
    outs = [t.reduce_received(M, N) for t in ranks]
    torch.cuda.synchronize()
    for q, y in enumerate(outs):
        ref = full[q * rows:(q + 1) * rows]
        assert (y.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 2e-2, q
    ranks[0].close()
