"""Receive-row layout of the GPU expert-parallel MoE: every (source, expert) block lands in a
disjoint row range of its holder, experts contiguous and in expert order, sources in rank order."""

import random

from resihp_megatron_b200.parallel.moe_ep import receive_layout


def test_receive_rows_tile_each_holder_buffer():
    rng = random.Random(0)
    for world, E in ((4, 8), (8, 8), (2, 6), (3, 7)):
        holder = [e * world // E for e in range(E)]
        table = [[rng.randrange(0, 50) for _ in range(E)] for _ in range(world)]
        for h in range(world):
            rows = []
            for src in range(world):
                rowbase, _ = receive_layout(table, holder, src, world)
                for e in range(E):
                    if holder[e] == h:
                        rows.append((rowbase[e], rowbase[e] + table[src][e], e, src))
            rows.sort()
            pos = 0
            for a, b, e, src in rows:
                assert a == pos, (world, E, h)
                pos = b
            _, ranges = receive_layout(table, holder, h, world)
            assert sum(n for _, n in ranges) == pos
            # expert-major, then source order
            assert [(e, src) for _, _, e, src in rows] == sorted((e, src) for _, _, e, src in rows)


def test_replica_cycles_deal_positions_onto_disjoint_rows():
    """Replicated experts: the dispatch kernel's row formula (rowbase[e][h] + (p // L) * slots of h
    per cycle + rank of the slot) maps every position dealt to holder h onto its block exactly."""
    from resihp_megatron_b200.parallel.moe_ep import replica_cycles, replica_layout

    rng = random.Random(1)
    world, E = 4, 5
    holders = [[0, 1], [1], [2, 3, 0], [3], [0]]
    cycles = replica_cycles(holders, {1: 0.5, 3: 1.5})
    assert all(set(c) == set(h) for c, h in zip(cycles, holders))
    table = [[rng.randrange(0, 40) for _ in range(E)] for _ in range(world)]
    filled = {h: [] for h in range(world)}
    for src in range(world):
        rowbase, _ = replica_layout(table, cycles, src, world)
        for e in range(E):
            L = len(cycles[e])
            for p in range(table[src][e]):
                j = p % L
                h = cycles[e][j]
                row = rowbase[e][h] + (p // L) * cycles[e].count(h) + cycles[e][:j].count(h)
                filled[h].append(row)
    for h in range(world):
        _, ranges = replica_layout(table, cycles, h, world)
        total = sum(n for _, n in ranges)
        assert sorted(filled[h]) == list(range(total)), h
