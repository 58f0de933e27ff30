"""Peer-to-peer state migration (``parallel.migration``): a TP2 -> TP1 reshard of a row-parallel
weight (column blocks: strided copies), a column-parallel weight (row blocks) and a replicated
vector, for three kinds, between two emulated ranks on one GPU; the result must equal the
logical tensors bit for bit."""

import pytest
import torch

pytestmark = pytest.mark.gpu

KINDS = ("param", "exp_avg", "exp_avg_sq")


def test_p2p_migration_tp2_to_tp1_is_exact():
    from resihp_megatron_b200.parallel.migration import migrate_p2p, pack_table
    from resihp_megatron_b200.parallel.symm import SymmetricHeap
    from resihp_megatron_b200.state.layer_registry import FULL, TensorSpec
    from resihp_megatron_b200.state.transfer_plan import plan_transfers

    specs = {"w_row": TensorSpec("w_row", (64, 256), 1), "w_col": TensorSpec("w_col", (256, 64), 0),
             "norm": TensorSpec("norm", (64,), None)}
    g = torch.Generator(device="cuda").manual_seed(0)
    full = {k: {key: torch.randn(s.global_shape, device="cuda", generator=g) for key, s in specs.items()}
            for k in KINDS}
    halves = [(0, 128), (128, 256)]
    old_h = {"w_row": [("d0", halves[0]), ("d1", halves[1])], "w_col": [("d0", halves[0]), ("d1", halves[1])],
             "norm": [("d0", FULL), ("d1", FULL)]}
    new_h = {"w_row": [("d0", (0, 256))], "w_col": [("d0", (0, 256))], "norm": [("d0", FULL)]}
    world = ["d0", "d1"]

    def local(d):
        out = {k: {} for k in KINDS}
        for key, hs in old_h.items():
            for dev, iv in hs:
                if dev == d:
                    s = specs[key]
                    for k in KINDS:
                        t = full[k][key]
                        out[k][key] = t if s.dim is None else t.narrow(s.dim, iv[0], iv[1] - iv[0]).contiguous()
        return out

    tplan = plan_transfers(old_h, new_h, valid_sources=set(world), node_of={"d0": "n0", "d1": "n0"})
    cap = max(pack_table(old_h, d, specs, KINDS)[1] for d in world)
    heaps = SymmetricHeap.emulated({"stage": (cap // 4, torch.float32)}, 2, "cuda")
    kw = dict(specs=specs, old_h=old_h, new_h=new_h, kinds=KINDS, device="cuda")
    for r, d in enumerate(world):
        migrate_p2p(tplan, d, world, old_state=local(d), new_state=None, _heap=heaps[r], _copy=False, **kw)
    new_state = {k: {key: torch.full(s.global_shape, float("nan"), device="cuda") for key, s in specs.items()}
                 for k in KINDS}
    pulled = migrate_p2p(tplan, "d0", world, old_state=None, new_state=new_state, _heap=heaps[0], _stage=False, **kw)
    torch.cuda.synchronize()
    for k in KINDS:
        for key in specs:
            assert torch.equal(new_state[k][key], full[k][key]), (k, key)
    assert pulled == sum(4 * t.numel() for t in full["param"].values()) * len(KINDS)
    heaps[0].close()


def test_fused_heterogeneous_tp_gradient_reduction_emulated():
    """Replicas of one stage with different TP degrees (TP2 on ranks 0-1, TP1 on rank 2), emulated
    on one GPU: each rank packs its slices of every holder set into its heap region, sums the set
    from every holder's region in rank order and unpacks -- every interval of every sharded tensor
    ends up as the sum of the two replicas' gradients, bit-identical on its two holders."""
    from resihp_megatron_b200.models.config import GPTConfig
    from resihp_megatron_b200.models.params import FlatParams
    from resihp_megatron_b200.models.tp_stage import stage_param_specs
    from resihp_megatron_b200.parallel.symm import SymmetricHeap
    from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan, StageGroup
    from resihp_megatron_b200.runtime.gpu_runtime import HeteroFusedSync

    cfg = GPTConfig(name="h", vocab_size=256, hidden=256, layers=2, heads=4, kv_heads=2, ffn=512, seq_len=128)
    ids = ("d0", "d1", "d2")
    groups = (StageGroup(0, 0, ids[0:2], (0, 2)), StageGroup(1, 0, ids[2:3], (0, 2)))
    plan = HeteroParallelPlan(1, ids, 2, 1, 2, groups, 2, ((0, 1),), sequence_parallel=True)
    layouts = [(0, 2), (1, 2), (0, 1)]  # (tp rank, tp size) of ranks 0, 1, 2
    params = []
    for tr, ts in layouts:
        _, shd = stage_param_specs(cfg, range(2), True, True, tr, ts)
        P = FlatParams(shd, "cuda")
        params.append(P)
    # the "full" gradient of each replica; each rank holds its shard of its replica's gradient
    torch.manual_seed(0)
    full = [{n: torch.randn(P.specs[n].full_shape or P.specs[n].shape, device="cuda") for n in params[2].order}
            for _ in range(2)]
    for r, P in enumerate(params):
        rep = 0 if r < 2 else 1
        for n in P.order:
            s = P.specs[n]
            P.g(n).copy_(full[rep][n].narrow(s.shard_dim, s.shard_range[0], s.shard_range[1] - s.shard_range[0]))
    # emulated heaps need their size up front: every rank's shard is an upper bound of its regions
    segs = {"region": (max(P.numel for P in params) + 1024, torch.float32)}
    heaps = SymmetricHeap.emulated(segs, 3, "cuda")
    syncs = [HeteroFusedSync(plan, 0, r, None, "cuda", _heap=heaps[r], _ranks=(0, 1, 2)) for r in range(3)]
    for s_, P in zip(syncs, params):
        s_.attach(P)
        assert s_.fused
    for s_ in syncs:
        s_.pack()
    for s_ in syncs:
        s_.sum()
    for s_ in syncs:
        s_.unpack()
    torch.cuda.synchronize()
    for r, P in enumerate(params):
        for n in P.order:
            s = P.specs[n]
            want = (full[0][n] + full[1][n]).narrow(s.shard_dim, s.shard_range[0], s.shard_range[1] - s.shard_range[0])
            assert torch.equal(P.g(n), want), (r, n)
    heaps[0].close()
