"""Host side of the peer-to-peer state migration (``parallel.migration``): staging offsets and the
strided-copy pieces of a TP2 -> TP1 reshard, executed by a byte-level stand-in for the copy
kernel on host memory.  The GPU test runs the same case on the kernel."""

import ctypes

import torch

KINDS = ("param", "exp_avg", "exp_avg_sq")


class _HostHeap:
    """Two ranks' staging areas in host memory, shaped like the symmetric heap's interface."""

    def __init__(self, bufs, rank):
        self.bufs, self.rank = bufs, rank

    def tensor(self, name):
        return self.bufs[self.rank]

    def peer_ptrs(self, name):
        return [b.data_ptr() for b in self.bufs]


def _copy2d(six, device):
    for i in range(0, len(six), 6):
        src, dst, rows, row_bytes, sp, dp = six[i:i + 6]
        assert row_bytes % 16 == 0 and sp % 16 == 0 and dp % 16 == 0
        for r in range(rows):
            ctypes.memmove(dst + r * dp, src + r * sp, row_bytes)


def test_pieces_reassemble_logical_tensors(monkeypatch):
    from resihp_megatron_b200.parallel import migration
    from resihp_megatron_b200.state.layer_registry import FULL, TensorSpec
    from resihp_megatron_b200.state.transfer_plan import plan_transfers

    class _Ext:
        symm_copy2d = staticmethod(_copy2d)

    monkeypatch.setattr(migration, "ext", lambda: _Ext)
    specs = {"w_row": TensorSpec("w_row", (64, 256), 1), "w_col": TensorSpec("w_col", (256, 64), 0),
             "norm": TensorSpec("norm", (64,), None)}
    g = torch.Generator().manual_seed(0)
    full = {k: {key: torch.randn(s.global_shape, generator=g) for key, s in specs.items()} for k in KINDS}
    halves = [(0, 128), (128, 256)]
    old_h = {"w_row": [("d0", halves[0]), ("d1", halves[1])], "w_col": [("d0", halves[0]), ("d1", halves[1])],
             "norm": [("d0", FULL), ("d1", FULL)]}
    new_h = {"w_row": [("d0", (0, 256))], "w_col": [("d0", (0, 256))], "norm": [("d0", FULL)]}
    world = ["d0", "d1"]
    tplan = plan_transfers(old_h, new_h, valid_sources=set(world), node_of={"d0": "n0", "d1": "n0"})
    cap = max(migration.pack_table(old_h, d, specs, KINDS)[1] for d in world)
    bufs = [torch.zeros(cap // 4) for _ in world]

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

    kw = dict(specs=specs, old_h=old_h, new_h=new_h, kinds=KINDS, device="cpu")
    for r, d in enumerate(world):
        migration.migrate_p2p(tplan, d, world, old_state=local(d), new_state=None, _heap=_HostHeap(bufs, r),
                              _copy=False, **kw)
    new_state = {k: {key: torch.full(s.global_shape, float("nan")) for key, s in specs.items()} for k in KINDS}
    migration.migrate_p2p(tplan, "d0", world, old_state=None, new_state=new_state, _heap=_HostHeap(bufs, 0),
                          _stage=False, **kw)
    for k in KINDS:
        for key in specs:
            assert torch.equal(new_state[k][key], full[k][key]), (k, key)
