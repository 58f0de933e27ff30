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
