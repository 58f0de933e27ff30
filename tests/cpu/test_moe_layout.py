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
