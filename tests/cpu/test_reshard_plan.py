"""The data-parallel reshard pull plan tiles every new optimizer shard exactly from the old
owners' shards, for shrinking and growing worlds."""

import pytest

from resihp_megatron_b200.parallel.dp_fused import reshard_pull_plan


@pytest.mark.parametrize("old_world,new_world", [(8, 7), (2, 1), (4, 3), (3, 4), (8, 5)])
def test_pull_plan_covers_new_shards(old_world, new_world):
    quantum = 128
    used = 1000 * quantum + 77
    old_numel = -(-used // (quantum * old_world)) * quantum * old_world
    new_numel = -(-used // (quantum * new_world)) * quantum * new_world
    old_shard, new_shard = old_numel // old_world, new_numel // new_world
    OLD, NEW = 1 << 40, 1 << 44
    old_ptrs = {k: [OLD + j * (1 << 36) + o * (1 << 32) for o in range(old_world)]
                for j, k in enumerate(("master", "exp_avg", "exp_avg_sq"))}
    for r in range(new_world):
        lo, hi = r * new_shard, (r + 1) * new_shard
        new_ptrs = {k: NEW + j * (1 << 36) for j, k in enumerate(("master", "exp_avg", "exp_avg_sq"))}
        t = reshard_pull_plan(old_world, old_shard, old_ptrs, lo, hi, new_ptrs, old_numel)
        triples = [t[i:i + 3] for i in range(0, len(t), 3)]
        for j, k in enumerate(("master", "exp_avg", "exp_avg_sq")):
            covered = []
            for src, dst, nbytes in triples:
                if not (NEW + j * (1 << 36) <= dst < NEW + (j + 1) * (1 << 36)):
                    continue
                d0 = (dst - new_ptrs[k]) // 4
                o = (src - OLD - j * (1 << 36)) >> 32
                s0 = (src - old_ptrs[k][o]) // 4 + o * old_shard
                assert s0 == lo + d0, "element i of the global flat space lands at position i - lo"
                covered.append((d0, d0 + nbytes // 4))
            covered.sort()
            want_hi = min(hi, old_numel) - lo
            pos = 0
            for a, b in covered:
                assert a == pos
                pos = b
            assert pos == max(0, want_hi)
