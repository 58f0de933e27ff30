"""Layout invariants of the symmetric peer heap (host side): one signal slot per rank, aligned,
non-overlapping segments inside the region, for random segment sets and world sizes."""

import random

import pytest
import torch


def test_layout_invariants_hold_for_random_segment_sets():
    from resihp_megatron_b200.parallel.symm import ALIGN, SIGNAL_SLOT_BYTES, check_layout, layout

    rng = random.Random(0)
    dtypes = [torch.float32, torch.bfloat16, torch.int32, torch.uint8, torch.int64]
    for _ in range(200):
        world = rng.randint(1, 16)
        segs = {f"s{i}": (rng.randint(1, 10 ** 6), rng.choice(dtypes)) for i in range(rng.randint(1, 8))}
        out, pad, total = layout(segs, world)
        check_layout(out, pad, total, world)
        assert pad >= world * SIGNAL_SLOT_BYTES and total % ALIGN == 0


def test_check_layout_rejects_overlap_and_misalignment():
    from resihp_megatron_b200.parallel.symm import Segment, check_layout

    with pytest.raises(AssertionError):
        check_layout({"a": Segment(256, 100, torch.float32), "b": Segment(512, 10, torch.float32)}, 256, 4096, 2)
    with pytest.raises(AssertionError):
        check_layout({"a": Segment(300, 4, torch.float32)}, 256, 4096, 2)
    with pytest.raises(AssertionError):
        check_layout({"a": Segment(256, 10 ** 6, torch.float32)}, 256, 4096, 2)
