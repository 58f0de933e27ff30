"""Index arithmetic of the fused heterogeneous-TP reduction (``HeteroFusedSync.layout``), on the
CPU: replicas of one stage with TP2 and TP1 (and TP4 / TP2); every interval of every sharded
tensor lies in exactly one holder set with one holder per replica, every holder of a set agrees on
its size and places it at a region offset the others compute for it, a rank's regions do not
overlap, and each rank's pieces cover exactly its shared part of every shard."""

import pytest
import torch

from resihp_megatron_b200.models.config import GPTConfig
from resihp_megatron_b200.models.params import FlatParams
from resihp_megatron_b200.models.tp_stage import stage_param_specs
from resihp_megatron_b200.plan.hetero_plan import HeteroParallelPlan, StageGroup
from resihp_megatron_b200.runtime.gpu_runtime import HeteroFusedSync

CFG = GPTConfig(name="h", vocab_size=256, hidden=256, layers=2, heads=4, kv_heads=4, ffn=512, seq_len=128)


@pytest.mark.parametrize("tps", [(2, 1), (4, 2), (2, 2, 1)])
def test_holder_sets_regions_and_pieces(tps):
    ids, groups, start = [], [], 0
    for rep, tp in enumerate(tps):
        devs = tuple(f"d{start + i}" for i in range(tp))
        ids += devs
        groups.append(StageGroup(rep, 0, devs, (0, CFG.layers)))
        start += tp
    plan = HeteroParallelPlan(1, tuple(ids), CFG.layers, 1, len(tps), tuple(groups), len(tps),
                              (tuple(range(len(tps))),), sequence_parallel=True)
    ranks = tuple(range(len(ids)))
    layouts = [(i, tp) for tp in tps for i in range(tp)]
    outs = []
    for r, (tr, ts) in enumerate(layouts):
        _, shd = stage_param_specs(CFG, range(CFG.layers), True, True, tr, ts)
        P = FlatParams(shd, "cpu")
        sync = HeteroFusedSync(plan, 0, r, None, "cpu", _ranks=ranks)
        super(HeteroFusedSync, sync).attach(P)  # the holder-set slices of this rank
        outs.append((P, sync, sync.layout(P)))
    sets, size, offsets, totals, _ = outs[0][2]
    # every rank computes the same sets, sizes and offsets
    for _, _, (s2, z2, o2, t2, _) in outs:
        assert s2 == sets and z2 == size and o2 == offsets and t2 == totals
    # one holder per replica in every set; every interval of every sharded tensor in exactly one set
    rep_of = {r: next(i for i, g in enumerate(groups) if ids[r] in g.devices) for r in ranks}
    for h in sets:
        assert sorted(rep_of[r] for r in h) == list(range(len(tps)))
    P0 = outs[0][0]
    for name in P0.order:
        sp = P0.specs[name]
        if sp.shard_dim is None:
            continue
        covered = sorted((lo, lo + ln) for h, pcs in sets.items() for nm, lo, ln in pcs if nm == name)
        edges = [0] + [b for _, b in covered]
        assert [a for a, _ in covered] == edges[:-1] and edges[-1] == sp.full_shape[sp.shard_dim]
    # regions of a rank are disjoint and inside its total
    for r in ranks:
        spans = sorted((offsets[r][h], offsets[r][h] + size[h]) for h in offsets[r])
        for (a0, b0), (a1, _) in zip(spans, spans[1:]):
            assert b0 <= a1
        assert all(b <= totals[r] for _, b in spans)
    # each rank's pieces: its shard's elements that another replica also holds, each exactly once
    for r, (P, sync, (_, _, _, _, geo)) in enumerate(outs):
        want = sum(size[h] for h in offsets[r])
        got = sum(rows * row_bytes // 4 for _, _, _, rows, row_bytes, _ in geo)
        assert got == want
        for h, poff, *_ in geo:
            assert 0 <= poff < size[h]
