"""Fused data-parallel step over real NVLink peers (2 GPUs, NCCL for the handshake): losses
and weights match the NCCL reduce-scatter / all-gather path, and every rank holds identical
weights.  Skipped with fewer than 2 GPUs."""

import os

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.train.gpu_trainer import GPUTrainer

    out = {}
    for impl in ("fused", "nccl"):
        tr = GPUTrainer(TINY, global_batch=4, micro_batch=1, seq_len=256, lr=1e-3, dp_group=dist.group.WORLD,
                        dp_impl=impl)
        g = torch.Generator().manual_seed(5)
        losses = []
        for _ in range(3):
            ids = torch.randint(0, TINY.vocab_size, (4, 257), generator=g)
            lo = rank * 2
            x = ids[lo:lo + 2, :-1].contiguous().pin_memory()
            y = ids[lo:lo + 2, 1:].contiguous().pin_memory()
            losses.append(tr.train_step(x, y))
        w = tr.model.params.bf16.float().cpu()
        out[impl] = (losses, w)
        tr.close()
    dist.barrier()
    dist.destroy_process_group()
    import io

    buf = io.BytesIO()  # bytes, not shared-memory tensors: the child exits before the parent reads
    torch.save((rank, out["fused"][0], out["nccl"][0], out["fused"][1], out["nccl"][1]), buf)
    q.put(buf.getvalue())


def test_fused_dp_matches_nccl_path_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from tests.dist_utils import free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        import io

        r, lf, ln, wf, wn = torch.load(io.BytesIO(q.get(timeout=600)))
        res[r] = (lf, ln, wf, wn)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        lf, ln, wf, wn = res[r]
        assert lf == pytest.approx(ln, rel=2e-3)
        assert (wf - wn).abs().max().item() < 5e-2
    assert torch.equal(res[0][2], res[1][2]), "fused path: identical weights on every rank"


def _shrink_worker(rank, world, port, q):
    import io

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.train.gpu_trainer import GPUTrainer

    g = torch.Generator().manual_seed(9)
    batches = [torch.randint(0, TINY.vocab_size, (4, 257), generator=g) for _ in range(3)]

    def local(tr, b):
        lo = tr.batch_offset
        return (b[lo:lo + tr.local_batch, :-1].contiguous().pin_memory(),
                b[lo:lo + tr.local_batch, 1:].contiguous().pin_memory())

    results = {}
    for mode in ("steady", "shrink"):
        tr = GPUTrainer(TINY, global_batch=4, micro_batch=2, seq_len=256, lr=1e-3, dp_group=dist.group.WORLD,
                        spare_bank=True)
        losses = [tr.train_step(*local(tr, b)) for b in batches[:2]]
        group = dist.new_group([0])
        alive = True
        if mode == "shrink":
            alive = tr.shrink([0], group)
        if alive:
            losses.append(tr.train_step(*local(tr, batches[2])))
            results[mode] = (losses, tr.model.params.bf16.float().cpu())
        if alive:
            tr.close()
        dist.barrier()
    dist.destroy_process_group()
    buf = io.BytesIO()
    torch.save((rank, results), buf)
    q.put(buf.getvalue())


def test_live_shrink_migrates_optimizer_state_over_nvlink():
    """2 ranks train, rank 1 leaves between steps, its optimizer shard is pulled peer to peer into
    rank 0's new layout, and the next step equals the step of the unchanged 2-rank job."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import io

    import torch.multiprocessing as mp

    from tests.dist_utils import free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_shrink_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, out = torch.load(io.BytesIO(q.get(timeout=600)))
        res[r] = out
    for p in procs:
        p.join(timeout=60)
    steady, shrunk = res[0]["steady"], res[0]["shrink"]
    assert "shrink" not in res[1], "the departing rank stops"
    assert shrunk[0][:2] == steady[0][:2]
    assert shrunk[0][2] == pytest.approx(steady[0][2], rel=2e-3)
    assert (shrunk[1] - steady[1]).abs().max().item() < 2e-2
