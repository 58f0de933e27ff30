"""ResilientCommManager on gloo ranks: generation build in both subgroup modes with validation,
survivor rebuild after a rank exits between steps, and abort latency (a rank blocked in a
collective that a peer never joins leaves it within 2 s of ``abort()``), plus the abort hooks."""

import pytest

from tests.dist_utils import spawn

pytestmark = pytest.mark.dist


def _build(rank, world, port, store_addr, mode):
    import torch
    import torch.distributed as dist

    from resihp_megatron_b200.comm.comm_manager import ResilientCommManager
    from resihp_megatron_b200.comm.group_spec import GroupSpec

    ids = [f"w{i}" for i in range(world)]
    specs = [GroupSpec("tp/a", (0, 1), "tp"), GroupSpec("tp/b", (2, 3), "tp"), GroupSpec("dp", (0, 2), "dp"),
             GroupSpec("dp2", (1, 3), "dp")]
    mgr = ResilientCommManager("gloo", timeout_s=30, subgroup_mode=mode)
    comms = mgr.build(1, ids, ids[rank], specs, store_addr=store_addr, store_prefix=f"{mode}/gen1/")
    t = torch.ones(1)
    dist.all_reduce(t, group=comms.group("tp/a" if rank < 2 else "tp/b"))
    out = {"path": comms.path, "tp_sum": t.item(), "member_dp": comms.is_member("dp")}
    # rank 3 leaves between steps; the survivors build generation 2 without it
    if rank == world - 1:
        import os

        os._exit(0)
    comms2 = mgr.build(2, ids[:-1], ids[rank], [GroupSpec("pair", (0, 1), "dp")], store_addr=store_addr,
                       store_prefix=f"{mode}/gen2/")
    t = torch.ones(1)
    dist.all_reduce(t)
    out.update(path2=comms2.path, world2=t.item())
    mgr.destroy()
    return out


@pytest.mark.parametrize("mode", ["local", "split"])
def test_generation_build_validate_and_survivor_rebuild(store, mode):
    res = spawn(_build, 4, store, mode, timeout=180, expect_dead={3})
    assert sorted(res) == [0, 1, 2]
    for r, out in res.items():
        assert out["path"] == "fresh" and out["tp_sum"] == 2.0 and out["world2"] == 3.0
        assert out["member_dp"] == (r in (0, 2))


def _abort(rank, world, port, store_addr):
    import threading
    import time

    import torch
    import torch.distributed as dist

    from resihp_megatron_b200.comm.comm_manager import CommAborted, ResilientCommManager

    ids = [f"w{i}" for i in range(world)]
    mgr = ResilientCommManager("gloo", timeout_s=60)
    mgr.build(1, ids, ids[rank], [], store_addr=store_addr, store_prefix="abort/gen1/")
    hooked = []
    mgr.add_abort_hook(lambda: hooked.append(True))
    if rank == 1:  # never joins the collective below; waits for rank 0 to finish the test
        time.sleep(8)
        return {"rank": 1}
    t = torch.ones(1)
    work = dist.all_reduce(t, async_op=True)
    threading.Timer(1.0, mgr.abort).start()
    t0 = time.monotonic()
    try:
        mgr.guarded_wait(work, timeout=30, what="blocked all-reduce")
        aborted = False
    except CommAborted:
        aborted = True
    return {"aborted": aborted, "latency": time.monotonic() - t0, "hooked": bool(hooked)}


def test_abort_ends_a_blocked_collective_quickly(store):
    res = spawn(_abort, 2, store, timeout=120)
    out = res[0]
    assert out["aborted"] and out["hooked"]
    assert out["latency"] < 1.0 + 2.0, out


def _mismatched_generation(rank, world, port, store_addr):
    from resihp_megatron_b200.comm.comm_manager import GenerationBuildError, ResilientCommManager

    ids = [f"w{i}" for i in range(world)]
    mgr = ResilientCommManager("gloo", timeout_s=30)
    try:  # rank 1 is one transaction behind: it builds generation 4 while rank 0 builds 5
        mgr.build(5 - rank, ids, ids[rank], [], store_addr=store_addr, store_prefix="epoch/gen/")
        refused = False
    except GenerationBuildError:
        refused = True
    mgr.destroy()
    return {"refused": refused}


def test_generation_handshake_refuses_ranks_of_different_generations(store):
    """Every rank of a new world checks that all ranks build the same generation number."""
    res = spawn(_mismatched_generation, 2, store, timeout=120)
    assert res[0]["refused"] and res[1]["refused"], res
