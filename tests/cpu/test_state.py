"""State layer: sampler and RNG, transactions and roll-forward, Adam vs torch, snapshots,
resharding checkpoints, DP planner helpers, reference model invariants, transfer plans."""

import pytest
import torch

from resihp_megatron_b200.plan.dp_planner import assign_sources, weighted_assignment
from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan, StageGroup
from resihp_megatron_b200.runtime.optim import Adam
from resihp_megatron_b200.runtime.reference_model import (RefModelConfig, RefStage, full_layer_params, global_tokens,
                                                          microbatch, reference_train)
from resihp_megatron_b200.state.checkpoint import SliceCheckpointer, SliceMeta
from resihp_megatron_b200.state.layer_registry import (FULL, TensorSpec, device_layout, holdings,
                                                       reference_layer_of, reference_specs)
from resihp_megatron_b200.state.redundancy import HolderMap, HostSnapshotManager, distopt_twin_holders
from resihp_megatron_b200.state.rng_data import IndexAddressableSampler, capture_rng_state, generator, restore_rng_state
from resihp_megatron_b200.state.transaction import TransactionManager, TxnPhase, roll_forward_plan
from resihp_megatron_b200.state.transfer_plan import plan_transfers


def test_sampler_deterministic_and_covers_an_epoch():
    s = IndexAddressableSampler(num_samples=20, global_batch_size=8, micro_batch_size=2, seed=3)
    assert s.num_microbatches == 4
    b0 = s.batch_indices(0)
    assert b0 == IndexAddressableSampler(20, 8, 2, seed=3).batch_indices(0)
    assert sum((s.microbatch_indices(0, m) for m in range(4)), []) == b0
    assert sorted(s.batch_indices(0) + s.batch_indices(1) + s.batch_indices(2)[:4]) == list(range(20))
    with pytest.raises(IndexError):
        s.microbatch_indices(0, 4)


def test_counter_rng_and_global_rng_restore():
    a = torch.rand(3, generator=generator(1, 2, 3))
    assert torch.equal(a, torch.rand(3, generator=generator(1, 2, 3)))
    assert not torch.equal(a, torch.rand(3, generator=generator(1, 2, 4)))
    st = capture_rng_state()
    x = torch.rand(4)
    restore_rng_state(st)
    assert torch.equal(x, torch.rand(4))


def test_transaction_lifecycle_and_rollback():
    txm = TransactionManager()
    txm.begin(0)
    txm.on_reduced()
    txm.on_step_begin()
    txm.on_commit()
    assert txm.committed_iteration == 0 and txm.cursor.iteration == 1
    txm.begin(1)
    st = torch.get_rng_state()
    torch.rand(10)
    info = txm.abort()
    assert torch.equal(torch.get_rng_state(), st)
    assert info == {"committed_iteration": 0, "has_reduced_grads": False, "inflight_iteration": 1}
    txm.discard()
    txm.begin(1)
    txm.on_reduced()
    txm.abort()
    assert txm.has_reduced_grads and txm.current.phase == TxnPhase.REDUCED
    with pytest.raises(ValueError):
        TransactionManager().begin(3)


def test_transaction_buffers_roll_back_unless_rolling_forward():
    amax = torch.ones(3)
    txm = TransactionManager(buffers=lambda: {"amax": amax})
    txm.begin(0)
    amax.add_(1)
    txm.abort()
    assert torch.equal(amax, torch.ones(3))
    txm.discard()
    txm.begin(0)
    amax.add_(5)
    txm.on_reduced()
    txm.abort()
    assert torch.equal(amax, torch.full((3,), 6.0))
    txm.discard()
    assert torch.equal(amax, torch.ones(3))
    txm.begin(0)
    amax.add_(2)
    txm.on_reduced()
    txm.on_step_begin()
    txm.on_commit()
    assert torch.equal(amax, torch.full((3,), 3.0))


def test_roll_forward_plan():
    rec = {"a": {"committed_iteration": 7, "has_reduced_grads": False},
           "b": {"committed_iteration": 6, "has_reduced_grads": True, "inflight_iteration": 7},
           "c": {"committed_iteration": 6, "has_reduced_grads": False, "inflight_iteration": 7}}
    p = roll_forward_plan(rec, ["a", "b", "c", "d"])
    assert p["target_iteration"] == 7
    assert p["up_to_date"] == ["a"] and p["local_step"] == ["b"] and p["needs_state"] == ["c", "d"]
    assert roll_forward_plan({}, ["x"])["up_to_date"] == ["x"]


def test_adam_bitwise_equal_to_torch():
    torch.manual_seed(0)
    w = torch.randn(5, 3, dtype=torch.float64)
    p1, p2 = torch.nn.Parameter(w.clone()), torch.nn.Parameter(w.clone())
    ours = Adam({"w": p1}, lr=0.01, weight_decay=0.1)
    ref = torch.optim.Adam([p2], lr=0.01, weight_decay=0.1, foreach=False)
    for i in range(5):
        g = torch.randn(5, 3, dtype=torch.float64)
        p1.grad, p2.grad = g.clone(), g.clone()
        ours.step()
        ref.step()
        assert torch.equal(p1, p2), i
    assert torch.equal(ours.state["w"]["exp_avg_sq"], ref.state[p2]["exp_avg_sq"])


def test_snapshots_and_holder_maps():
    snaps = HostSnapshotManager(interval=2)
    assert not snaps.due(0) and snaps.due(1)
    t = {"a": torch.ones(2)}
    snaps.snapshot(1, t)
    t["a"].add_(1)
    it, s = snaps.latest()
    assert it == 1 and torch.equal(s["a"], torch.ones(2))
    holders = distopt_twin_holders(["r0", "r1", "r2", "r3"], 2)
    assert holders == {"shard0": ["r0", "r2"], "shard1": ["r1", "r3"]}
    hm = HolderMap(holders)
    assert hm.lost({"r0"}) == [] and hm.lost({"r0", "r2"}) == ["shard0"]
    assert hm.node_diverse({"r0": "n0", "r1": "n0", "r2": "n1", "r3": "n1"}.get)
    assert not hm.node_diverse({"r0": "n0", "r1": "n1", "r2": "n0", "r3": "n1"}.get)
    with pytest.raises(ValueError):
        distopt_twin_holders(["a", "b", "c"], 2)


def test_checkpoint_format_and_reshard_on_load(tmp_path):
    ck = SliceCheckpointer(tmp_path)
    full = torch.arange(24, dtype=torch.float64).reshape(6, 4)
    for r, (a, b) in enumerate([(0, 2), (2, 4), (4, 6)]):
        ck.save(5, f"w{r}", [(SliceMeta("W", (6, 4), 0, (a, b)), {"param": full[a:b], "m": -full[a:b]}),
                             (SliceMeta("b", (4,), None, (0, 1)), {"param": torch.ones(4), "m": torch.zeros(4)})],
                blocking=True)
    d = tmp_path / "iter_00000005"
    assert (d / "w0.pt").exists() and (d / "w0.done").exists() and not list(d.glob(".*.tmp"))
    assert ck.latest_complete({"W": ((6, 4), 0), "b": ((4,), None)}) == 5
    got = ck.load(5, [SliceMeta("W", (6, 4), 0, (1, 5)), SliceMeta("b", (4,), None, (0, 1))], kinds=("param", "m"))
    assert torch.equal(got["W"]["param"], full[1:5]) and torch.equal(got["W"]["m"], -full[1:5])
    assert torch.equal(got["b"]["param"], torch.ones(4))
    assert not ck.complete(5, {"W": ((8, 4), 0)})
    with pytest.raises(KeyError):
        ck.load(5, [SliceMeta("W", (8, 4), 0, (5, 8))], kinds=("param",))


def test_dp_planner_helpers():
    a = weighted_assignment(["a", "b", "c"], 8, {"a": 1.0, "b": 1.0, "c": 0.5})
    assert sorted(sum(a.values(), [])) == list(range(8)) and len(a["c"]) < len(a["a"])
    src = assign_sources(["x", "y", "z"], ["p", "q"], {"x": "n0", "y": "n1", "z": "n1", "p": "n1", "q": "n2"})
    assert src["y"] == "p" and set(src) == {"x", "y", "z"}


def test_reference_model_is_partition_invariant():
    cfg = RefModelConfig()
    full = full_layer_params(cfg, 2)
    stage = RefStage(cfg, 1, 3)
    assert set(stage.named_state()) == {f"layers.{l}.{k}" for l in (1, 2) for k in full}
    assert torch.equal(stage.named_state()["layers.2.fc1.weight"], full["fc1.weight"])
    s = IndexAddressableSampler(64, 8, 2, seed=1)
    m = microbatch(cfg, s, 0, 1)
    assert m.x.shape[0] % cfg.token_multiple == 0 and m.num_tokens == sum(m.doc_lengths)
    assert global_tokens(cfg, s, 0) == sum(microbatch(cfg, s, 0, k).num_tokens for k in range(4))
    losses, _ = reference_train(cfg, s, 3)
    assert losses[-1] < losses[0]
    fp8, state = reference_train(RefModelConfig(amax_history=4), s, 3)
    assert fp8 != losses and state["layers.0.amax_history"][0] > 0


def _plan(groups, layers=4, M=4):
    world = tuple(d for g in groups for d in g.devices)
    S = max(g.stage for g in groups) + 1
    R = max(g.replica for g in groups) + 1
    rows = tuple(tuple(min(m * R // M, R - 1) for m in range(M)) for _ in range(S))
    return HeteroParallelPlan(1, world, layers, S, R, tuple(groups), M, rows)


def _covered(tp, new_h):
    for key, hs in new_h.items():
        for dst, iv in hs:
            pieces = sorted([o for d, k, o in tp.reuse if d == dst and k == key]
                            + [t.interval for t in tp.transfers if t.dst == dst and t.key == key])
            pos = iv[0]
            for a, b in pieces:
                assert a == pos, (key, dst, pieces, iv)
                pos = b
            assert pos == iv[1]


def test_transfer_plan_tp_shrink_and_layer_move():
    specs = reference_specs(RefModelConfig())
    old = _plan([StageGroup(0, 0, ("a", "b"), (0, 2)), StageGroup(0, 1, ("c", "d"), (2, 4)),
                 StageGroup(1, 0, ("e", "f"), (0, 2)), StageGroup(1, 1, ("g", "h"), (2, 4))])
    new = _plan([StageGroup(0, 0, ("a", "b"), (0, 3)), StageGroup(0, 1, ("c",), (3, 4)),
                 StageGroup(1, 0, ("e", "f"), (0, 3)), StageGroup(1, 1, ("g", "h"), (3, 4))])
    old_h, new_h = holdings(old, specs, reference_layer_of), holdings(new, specs, reference_layer_of)
    nodes = {"a": "n0", "b": "n0", "c": "n1", "d": "n1", "e": "n2", "f": "n2", "g": "n3", "h": "n3"}
    tp = plan_transfers(old_h, new_h, valid_sources=set(old.world) - {"d"}, node_of=nodes)
    assert not tp.lost
    _covered(tp, new_h)
    assert all(t.src != "d" for t in tp.transfers)
    assert ("a", "layers.0.fc1.weight", (0, 12)) in tp.reuse
    c3 = [t for t in tp.transfers if t.key == "layers.3.fc1.weight" and t.dst == "c"]
    assert [t.interval for t in c3] == [(12, 24)] and c3[0].src in {"g", "h"}


def test_transfer_plan_locality_striping_and_lost():
    spec = {"w": TensorSpec("w", (16, 4), 0)}
    old = {"w": [("r0", (0, 16)), ("r1", (0, 16)), ("r2", (0, 16))]}
    nodes = {"r0": "n0", "r1": "n1", "r2": "n1", "x": "n1"}
    tp = plan_transfers(old, {"w": [("x", (0, 16))]}, valid_sources={"r0", "r1", "r2"}, node_of=nodes, chunk=4)
    assert [t.interval for t in tp.transfers] == [(0, 4), (4, 8), (8, 12), (12, 16)]
    assert {t.src for t in tp.transfers} == {"r1", "r2"}
    assert [t.src for t in plan_transfers(old, {"w": [("x", (0, 16))]}, valid_sources={"r0"},
                                          node_of=nodes).transfers] == ["r0"]
    tp3 = plan_transfers(old, {"w": [("x", (0, 16))], "v": [("x", FULL)]}, valid_sources=set(), node_of=nodes)
    assert ("w", (0, 16)) in tp3.lost and ("v", FULL) in tp3.lost
    assert tp.bytes_moved(spec, 2, 3) == 16 * 4 * 2 * 3
    lay = device_layout(holdings(_plan([StageGroup(0, 0, ("a", "b", "c"), (0, 4))]), reference_specs(RefModelConfig()),
                                 reference_layer_of), "b")
    assert lay["layers.1.fc1.weight"] == (8, 16) and lay["layers.1.ln.weight"] == FULL
