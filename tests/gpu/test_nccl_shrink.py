"""NCCL generation rebuild on 2-4 GPUs: the last rank leaves between steps (nothing of it in
flight), the survivors shrink the NCCL world (``dist.shrink_group``, NCCL >= 2.27.3) or build a
fresh one, validate every group and keep training collectives working.  Child processes, one
per GPU, with NVLS off."""

import os

import pytest
import torch

from tests.dist_utils import spawn

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, port, store_addr):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    from resihp_megatron_b200.comm.comm_manager import ResilientCommManager
    from resihp_megatron_b200.comm.group_spec import GroupSpec

    torch.cuda.set_device(rank)
    ids = [f"g{i}" for i in range(world)]
    mgr = ResilientCommManager("nccl", device=f"cuda:{rank}", timeout_s=60, validate_timeout_s=30)
    specs = [GroupSpec("pairs0", tuple(range(0, world, 2)), "dp")]
    mgr.build(1, ids, ids[rank], specs, store_addr=store_addr, store_prefix="shrink/gen1/")
    t = torch.ones(1, device="cuda")
    dist.all_reduce(t)
    torch.cuda.synchronize()
    first = t.item()
    dist.barrier()
    torch.cuda.synchronize()
    if rank == world - 1:
        os._exit(0)  # leaves between steps
    comms = mgr.build(2, ids[:-1], ids[rank], [], store_addr=store_addr, store_prefix="shrink/gen2/")
    t = torch.ones(1, device="cuda")
    dist.all_reduce(t)
    torch.cuda.synchronize()
    out = {"first": first, "second": t.item(), "path": comms.path}
    mgr.destroy()
    return out


def test_survivors_rebuild_nccl_without_the_leaver(store):
    n = min(4, torch.cuda.device_count())
    res = spawn(_worker, n, store, timeout=300, expect_dead={n - 1})
    assert sorted(res) == list(range(n - 1))
    for out in res.values():
        assert out["first"] == n and out["second"] == n - 1
        assert out["path"] in ("shrink", "fresh")
