"""The heterogeneous hybrid runtime on gloo ranks, each path checked against an independent
ground truth: pipeline-boundary routing against the rows a brute force says each receiver
needs, shard-aligned gradient sync against the dense sum of every replica's gradient, and whole
heterogeneous pipelines (stage-level migration, SP, zero bubble, interleaving, CP) against the
single-process float64 reference model."""

import itertools

import pytest
import torch

from tests.dist_utils import spawn

pytestmark = pytest.mark.dist

PAIRS = [(1, 1), (2, 1), (1, 3), (4, 2), (2, 3), (3, 4), (4, 3)]  # (sender TP, receiver TP)
ROWS = 24


def _routing(rank, world, port, store_addr):
    from resihp_megatron_b200.comm.comm_manager import ResilientCommManager
    from resihp_megatron_b200.comm.group_spec import GroupSpec
    from resihp_megatron_b200.comm.p2p import P2PEngine, boundary_routes, channel_name
    from resihp_megatron_b200.utils.intervals import even_split

    ids = [f"w{i}" for i in range(world)]
    specs = [GroupSpec(f"recv/{a}-{b}", tuple(range(a, a + b)), "tp") for a, b in PAIRS if b > 1]
    channel_pairs = sorted({(r.src, r.dst) for r in boundary_routes((0, 1, 2, 3), (4, 5, 6), ROWS)})
    specs += [GroupSpec(channel_name(s, d), (min(s, d), max(s, d)), "p2p") for s, d in channel_pairs]
    mgr = ResilientCommManager("gloo", timeout_s=30)
    comms = mgr.build(1, ids, ids[rank], specs, store_addr=store_addr, store_prefix="routing/gen1/")
    payload = torch.randn(ROWS, 5, generator=torch.Generator().manual_seed(3), dtype=torch.float64)
    checks = []

    def rows_of(ranks, r):  # brute force: which rows rank r owns in a group of len(ranks)
        return slice(*even_split(ROWS, len(ranks))[ranks.index(r)])

    for (a, b), sp in itertools.product(PAIRS, (False, True)):
        senders, receivers = tuple(range(a)), tuple(range(a, a + b))
        engine = P2PEngine(rank, mgr)
        tag = 1000 * sp + 10 * a + b
        posted = engine.send(payload[rows_of(senders, rank)] if sp else payload, senders, receivers, ROWS, sp,
                             tag) if rank in senders else []
        if rank in receivers:
            got = engine.recv(ROWS, (5,), torch.float64, senders, receivers, sp, tag,
                              tp_group=comms.group(f"recv/{a}-{b}") if b > 1 else None)
            checks.append(torch.equal(got, payload[rows_of(receivers, rank)] if sp else payload))
        engine.wait_sends(posted)
    channels = {(s, d): comms.group(channel_name(s, d)) for s, d in channel_pairs if rank in (s, d)}
    engine = P2PEngine(rank, mgr, channels=channels)
    posted = engine.send(payload, (0, 1, 2, 3), (4, 5, 6), ROWS, False, 7) if rank < 4 else []
    if 4 <= rank < 7:
        checks.append(torch.equal(engine.recv(ROWS, (5,), torch.float64, (0, 1, 2, 3), (4, 5, 6), False, 7,
                                              tp_group=comms.group("recv/4-3")), payload))
    engine.wait_sends(posted)
    mgr.destroy()
    return checks


def test_boundary_routing_delivers_exactly_the_needed_rows(store):
    results = spawn(_routing, 7, store, timeout=180)
    assert all(all(r) for r in results.values()) and sum(map(len, results.values())) > 20


def _grad_sync(rank, world, port, store_addr, sp):
    import zlib

    from resihp_megatron_b200.comm.comm_manager import ResilientCommManager
    from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan, StageGroup
    from resihp_megatron_b200.runtime.hetero_grad_sync import HeteroGradSync
    from resihp_megatron_b200.runtime.hetero_runtime import reference_partition_sizes, reference_shards
    from resihp_megatron_b200.runtime.reference_model import (PARAM_DIMS, RefModelConfig, RefStage, TPContext,
                                                              full_layer_params, shard)
    from resihp_megatron_b200.state.rng_data import generator

    cfg = RefModelConfig()
    ids = [f"w{i}" for i in range(world)]
    tp4, tp3 = StageGroup(0, 0, tuple(ids[:4]), (0, 1)), StageGroup(1, 0, tuple(ids[4:]), (0, 1))
    plan = HeteroParallelPlan(1, tuple(ids), 1, 1, 2, (tp4, tp3), 2, ((0, 1),), sequence_parallel=sp)
    mgr = ResilientCommManager("gloo", timeout_s=30)
    comms = mgr.build(1, ids, ids[rank], plan.group_specs(reference_partition_sizes(cfg)), store_addr=store_addr,
                      store_prefix=f"sync{int(sp)}/gen1/")
    replica = 0 if rank < 4 else 1
    group = (tp4, tp3)[replica]
    tp_rank = group.devices.index(ids[rank])
    tp = TPContext(group=comms.group(f"tp/r{replica}/s0"), rank=tp_rank, size=group.tp, sequence_parallel=sp,
                   waiter=mgr.guarded_wait)
    module = RefStage(cfg, 0, 1, tp)
    expected = {}
    for key, param in module.named_state().items():
        name = key.split(".", 2)[2]
        seed = zlib.crc32(name.encode())
        shape = full_layer_params(cfg, 0)[name].shape

        def dense(*parts):
            return torch.randn(shape, generator=generator(*parts, seed), dtype=cfg.dtype)

        # every replica's full gradient; the synced shard must be the sum over the replicas
        expected[key] = shard(dense(0) + dense(1), PARAM_DIMS[name], tp_rank, group.tp)
        mine = dense(replica)
        if module.sp_partial(key):  # partial sums over token shards that add up to ``mine``
            parts = [dense(replica, t, 5) for t in range(1, group.tp)]
            param.grad = mine - sum(parts) if tp_rank == 0 else parts[tp_rank - 1].clone()
        else:
            param.grad = shard(mine, PARAM_DIMS[name], tp_rank, group.tp)
    HeteroGradSync(plan, comms, mgr, 0, replica, module.named_state(), reference_shards(cfg, module),
                   tp_group=tp.group).sync()
    worst = max(float((p.grad - expected[k]).abs().max()) for k, p in module.named_state().items())
    mgr.destroy()
    return worst


@pytest.mark.parametrize("sp", [False, True])
def test_shard_aligned_sync_equals_the_dense_sum_tp4_with_tp3(store, sp):
    assert max(spawn(_grad_sync, 7, store, sp, timeout=180).values()) < 1e-12


# ---------------------------------------------------------------------- whole pipelines
def _scenario(name: str, ids: tuple, sp: bool):
    """(plan, model config) of a named heterogeneous layout."""
    from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan, StageGroup, interleave
    from resihp_megatron_b200.runtime.reference_model import RefModelConfig

    migrated = ((0, 0, 0, 0, 0, 1, 1, 1), (0, 0, 1, 1, 1, 1, 1, 1))  # stage-level micro-batch migration
    if name == "cp":  # cp = 2 everywhere; stage 0 has TP2 and TP1 replicas; replica 1 lost stage 1
        groups = (StageGroup(0, 0, ids[0:4], (0, 3), 2), StageGroup(1, 0, ids[4:6], (0, 3), 2),
                  StageGroup(0, 1, ids[6:8], (3, 4), 2))
        return HeteroParallelPlan(1, ids, 4, 2, 2, groups, 8, (migrated[0], (0,) * 8), sequence_parallel=sp), \
            RefModelConfig()
    split = 3 if name == "pipeline" else 5
    layers = 4 if name == "pipeline" else 8
    groups = (StageGroup(0, 0, ids[0:2], (0, split)), StageGroup(1, 0, ids[2:3], (0, split)),
              StageGroup(0, 1, ids[3:4], (split, layers)), StageGroup(1, 1, ids[4:7], (split, layers)))
    plan = HeteroParallelPlan(1, ids, layers, 2, 2, groups, 8, migrated, sequence_parallel=sp)
    return (interleave(plan, 2) if name == "interleaved" else plan), RefModelConfig(num_layers=layers)


def _train(rank, world, port, store_addr, name, sp, zb, iterations):
    from resihp_megatron_b200.comm.comm_manager import ResilientCommManager
    from resihp_megatron_b200.plan.ir import compute_order_to_ir, validate
    from resihp_megatron_b200.plan.simulator import schedule_with_fallback
    from resihp_megatron_b200.runtime.hetero_runtime import (HeteroRuntime, build_stage_module, channel_specs,
                                                             reference_partition_sizes)
    from resihp_megatron_b200.runtime.optim import Adam
    from resihp_megatron_b200.state.rng_data import IndexAddressableSampler

    ids = tuple(f"w{i}" for i in range(world))
    plan, cfg = _scenario(name, ids, sp)
    plan.validate()
    order = schedule_with_fallback(plan, lambda k, op, mb: 2.0 if op != "F" else 1.0, lambda a, b, kind: 0.1,
                                   split_backward=zb).order
    schedule = compute_order_to_ir(plan, order)
    validate(plan, schedule, split_backward=zb)
    mgr = ResilientCommManager("gloo", timeout_s=60)
    comms = mgr.build(1, list(ids), ids[rank], plan.group_specs(reference_partition_sizes(cfg))
                      + channel_specs(plan, schedule, 48), store_addr=store_addr,
                      store_prefix=f"{name}{int(sp)}{int(zb)}/gen1/")
    module = build_stage_module(cfg, plan, comms, mgr)
    optimizer = Adam(module.named_state(), lr=1e-2)
    runtime = HeteroRuntime(cfg, IndexAddressableSampler(256, 16, 2, seed=7), plan, schedule, comms, mgr, module,
                            use_channels=True)
    losses = []
    for it in range(iterations):
        losses.append(runtime.run_iteration(it))
        optimizer.step()
    me = ids[rank]
    group = plan.group_of_device(me)
    cp_slice = group.slice_of(me)
    result = {"losses": losses, "key": (group.replica, group.stage, cp_slice),
              "tp_rank": group.slice(cp_slice).index(me), "chunks": len(plan.groups_of_device(me)),
              "shards": {k: v.detach().clone() for k, v in module.named_state().items()}}
    mgr.destroy()
    return result


def _assert_matches_reference(results, cfg, iterations):
    from resihp_megatron_b200.runtime.reference_model import PARAM_DIMS, reference_train
    from resihp_megatron_b200.state.rng_data import IndexAddressableSampler

    losses, params = reference_train(cfg, IndexAddressableSampler(256, 16, 2, seed=7), iterations)
    assert all(r["losses"] == pytest.approx(losses, rel=1e-10) for r in results.values())
    by_group: dict = {}
    for r in results.values():
        by_group.setdefault(r["key"], []).append(r)
    seen = set()
    for members in by_group.values():  # reassemble each TP group's shards and compare to the full tensor
        members.sort(key=lambda r: r["tp_rank"])
        for key, first in members[0]["shards"].items():
            dim = PARAM_DIMS[key.split(".", 2)[2]]
            whole = first if dim is None else torch.cat([m["shards"][key] for m in members], dim=dim)
            torch.testing.assert_close(whole, params[key], rtol=1e-10, atol=1e-12)
            seen.add(key)
    assert seen == set(params)


@pytest.mark.parametrize("name,world,sp,zb", [
    ("pipeline", 7, False, False), ("pipeline", 7, True, False), ("pipeline", 7, False, True),
    ("pipeline", 7, True, True), ("interleaved", 7, False, False), ("interleaved", 7, True, True),
    ("cp", 8, False, False), ("cp", 8, True, False)])
def test_heterogeneous_pipeline_matches_the_float64_reference(store, name, world, sp, zb):
    from resihp_megatron_b200.runtime.reference_model import RefModelConfig

    results = spawn(_train, world, store, name, sp, zb, 3, timeout=240)
    if name == "interleaved":
        assert {r["chunks"] for r in results.values()} == {2}
    _assert_matches_reference(results, RefModelConfig(num_layers=8 if name == "interleaved" else 4), 3)
