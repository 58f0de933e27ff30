"""Symmetric peer memory on one GPU: the fused data-parallel step with emulated ranks against
an fp32 reference, and the bounded barrier's timeout and abort paths (a flag nothing sets; the
kernel returns a status, the context stays usable)."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fused_dp_step_emulated_ranks_matches_reference(tmp_path):
    from resihp_megatron_b200.ops._build import ext
    from resihp_megatron_b200.parallel.symm import SymmetricHeap

    from resihp_megatron_b200.detect.nccl_profile_reader import RingReader
    from resihp_megatron_b200.parallel.device_ring import DeviceRing

    W, n = 4, 1 << 16
    heaps = SymmetricHeap.emulated({"grad": (n, torch.float32), "weight": (n, torch.bfloat16)}, W, "cuda")
    for h in heaps:
        h.validate()
    import os

    ring_dir = tmp_path
    if os.path.isdir("/dev/shm"):  # tmpfs: registering its pages for device writes is supported
        import tempfile

        ring_dir = tempfile.mkdtemp(dir="/dev/shm")
    ring = DeviceRing(directory=str(ring_dir), capacity=16)
    torch.manual_seed(0)
    grads = [torch.randn(n, device="cuda") for _ in range(W)]
    for r, h in enumerate(heaps):
        h.tensor("grad").copy_(grads[r])
    master = torch.randn(n, device="cuda")
    shard = n // W
    lr, b1, b2, eps, wd, scale, step = 1e-2, 0.9, 0.95, 1e-8, 0.1, 0.5, 3
    m0 = torch.randn(n, device="cuda").abs() * 0.01
    v0 = torch.randn(n, device="cuda").abs() * 0.01
    states = []
    for r, h in enumerate(heaps):
        sl = slice(r * shard, (r + 1) * shard)
        st = [master[sl].clone(), m0[sl].clone(), v0[sl].clone()]
        ext().dp_step_fused(h.peer_ptrs("grad"), h.peer_ptrs("weight"), st[0], st[1], st[2], r * shard, lr, b1, b2,
                            eps, wd, False, step, scale, 0, ring.dev, ring.capacity, ring.stamp.data_ptr())
        states.append(st)
    torch.cuda.synchronize()
    # fp32 reference in the same formula order as torch.optim.Adam (L2 weight decay)
    g = sum(grads) * scale + wd * master
    m = m0 + (1 - b1) * (g - m0)
    v = v0 * b2 + (1 - b2) * g * g
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    p = master - lr / bc1 * (m / (v.sqrt() / bc2 ** 0.5 + eps))
    got = torch.cat([s[0] for s in states])
    torch.testing.assert_close(got, p, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(torch.cat([s[1] for s in states]), m, rtol=1e-5, atol=1e-7)
    for h in heaps:  # every rank received every shard
        assert torch.equal(h.tensor("weight"), got.bfloat16())
    # one device timing record per launch, readable by the NCCL-ring reader
    recs = RingReader(ring.path).poll()
    assert [r.func for r in recs] == ["dp_reduce_adam_gather"] * W
    assert all(r.end_ns > r.start_ns for r in recs) and all(r.count == shard for r in recs)
    ring.close()
    heaps[0].close()


def test_barrier_single_rank_then_timeout_and_abort_paths():
    from resihp_megatron_b200.parallel.symm import AbortWord, PeerAborted, PeerTimeout, SymmetricHeap

    one = SymmetricHeap({"x": (16, torch.float32)}, 0, 1, None, "cuda")
    one.barrier(1.0)
    one.barrier(1.0)
    one.check()
    one.close()
    # two emulated ranks, but only rank 0 ever arrives: its wait runs out and reports rank 1
    pair = SymmetricHeap.emulated({"x": (16, torch.float32)}, 2, "cuda")
    t0 = time.monotonic()
    pair[0].barrier(0.3)
    with pytest.raises(PeerTimeout, match="peer 1"):
        pair[0].check()
    assert time.monotonic() - t0 < 10
    # a failed barrier is sticky: the next one returns at once instead of waiting its budget
    t0 = time.monotonic()
    pair[0].barrier(30.0)
    with pytest.raises(PeerTimeout):
        pair[0].check()
    assert time.monotonic() - t0 < 5
    # the raised abort word ends the wait early
    abort = AbortWord()
    pair[0].abort = abort
    pair[0].status.zero_()
    abort.set()
    pair[0].barrier(30.0)
    t0 = time.monotonic()
    with pytest.raises(PeerAborted):
        pair[0].check()
    assert time.monotonic() - t0 < 5
    abort.close()
    from resihp_megatron_b200.ops.gemm import error_state

    error_state().zero_()  # the intended timeout recorded an error word
    x = torch.ones(4, device="cuda") * 2  # context still usable
    assert x.sum().item() == 8
    pair[0].close()


def test_vmm_region_exported_and_imported_aliases_the_same_memory():
    """A cuMem region exported as a file descriptor and imported again maps the same physical
    memory: writes through either mapping are seen through the other."""
    import os

    from resihp_megatron_b200.ops._build import ext

    p, fd, size = ext().vmm_alloc(1 << 20, 0)
    try:
        q = ext().vmm_import(fd, size, 0)
    finally:
        os.close(fd)
    n = size // 4
    a = ext().symm_tensor(p, n, "float32", 0)
    b = ext().symm_tensor(q, n, "float32", 0)
    assert p != q and int(a.abs().sum()) == 0  # zeroed at allocation
    a.copy_(torch.arange(n, device="cuda", dtype=torch.float32))
    torch.cuda.synchronize()
    assert torch.equal(b, a)
    b.fill_(3.0)
    torch.cuda.synchronize()
    assert bool((a == 3.0).all())
    del a, b
    ext().vmm_free(q, 0)
    ext().vmm_free(p, 0)


def test_vmm_heap_descriptor_exchange_between_two_ranks_in_threads():
    """Two heaps of one world built concurrently (threads standing in for processes) exchange
    their regions' descriptors over Unix sockets; each maps the other's region, a write by one is
    read through the other's mapping, and ``restrict`` drops the departed rank's mapping."""
    import threading

    from resihp_megatron_b200.parallel.symm import SymmetricHeap

    slots: list = [None, None]
    ready = threading.Barrier(2)

    def exchange_for(rank):
        def exchange(handle: bytes) -> list[bytes]:
            slots[rank] = handle
            ready.wait(timeout=30)
            return list(slots)
        return exchange

    heaps: list = [None, None]
    errors: list = []

    def build(rank):
        try:
            torch.cuda.set_device(0)
            heaps[rank] = SymmetricHeap({"x": (4096, torch.float32)}, rank, 2, exchange_for(rank), "cuda", alloc="vmm")
        except BaseException as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=build, args=(r,)) for r in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(60)
    assert not errors, errors
    h0, h1 = heaps
    h0.tensor("x").fill_(7.0)
    torch.cuda.synchronize()
    assert bool((h1.tensor("x", rank=0) == 7.0).all())
    h1.tensor("x").fill_(-1.0)
    torch.cuda.synchronize()
    assert bool((h0.tensor("x", rank=1) == -1.0).all())
    h0.restrict([0])
    assert h0.world == 1 and h0.bases == [h0.local_base]
    h0.close()
    h1.close()
