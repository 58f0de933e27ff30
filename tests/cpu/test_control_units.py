"""Units of the control plane and its helpers: the KV store (fake clock, leases, fenced
writes), health probes (fake NVML, a temporary sysfs tree), the fault grammar and injectors
(parse round trip, dry-run commands, device-setting gate, schedules), intervals, group-spec
layering and the ordering of generation hooks."""

import pytest

from resihp_megatron_b200.comm.group_spec import GroupSpec, canonical_order, split_layers
from resihp_megatron_b200.control.health import FATAL_XIDS, CompositeProbe, IBPortProbe, NVMLProbe
from resihp_megatron_b200.control.kvstore import InMemoryKV
from resihp_megatron_b200.inject.faults import (ExternalInjector, FaultInjector, FaultKind, parse_faults,
                                                run_schedule)
from resihp_megatron_b200.runtime.generation_hooks import CudaGraphHook, GenerationHooks, SymmetricHeapHook
from resihp_megatron_b200.utils import intervals as iv


class Clock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t


def test_kv_leases_cas_and_fenced_writes():
    clk = Clock()
    kv = InMemoryKV(clock=clk)
    lease = kv.grant_lease(1.0)
    assert kv.cas("leader", None, "c0", lease=lease)
    assert not kv.cas("leader", None, "c1")
    assert kv.put_if("state", "a", "leader", "c0") and kv.get("state") == "a"
    assert not kv.put_if("state", "b", "leader", "c1") and kv.get("state") == "a"
    clk.t = 0.8
    assert kv.keepalive(lease)
    clk.t = 1.7
    assert kv.get("leader") == "c0", "keepalive extended the lease"
    clk.t = 3.0
    assert kv.get("leader") is None and not kv.keepalive(lease), "an expired lease drops its keys"
    l2 = kv.grant_lease(1.0)
    assert kv.cas("leader", None, "c1", lease=l2)
    assert not kv.put_if("state", "late", "leader", "c0"), "the deposed leader is fenced"
    kv.put("ns/a", "1")
    kv.put("ns/b", "2")
    assert kv.get_prefix("ns/") == {"ns/a": "1", "ns/b": "2"}
    kv.revoke(l2)
    assert kv.get("leader") is None


class FakeEvent:
    def __init__(self, device, xid):
        self.device, self.eventData = device, xid


class FakeNVML:
    NVML_MEMORY_ERROR_TYPE_UNCORRECTED = 1
    NVML_VOLATILE_ECC = 0
    NVML_CLOCK_SM = 1
    NVML_TEMPERATURE_GPU = 0
    nvmlEventTypeXidCriticalError = 8

    def __init__(self, n=2):
        self.n = n
        self.pending = []
        self.ecc = [0] * n
        self.set_calls = 0

    def nvmlInit(self):
        pass

    def nvmlDeviceGetCount(self):
        return self.n

    def nvmlDeviceGetHandleByIndex(self, i):
        return ("h", i)

    def nvmlEventSetCreate(self):
        return "set"

    def nvmlDeviceRegisterEvents(self, h, mask, s):
        pass

    def nvmlEventSetWait(self, s, timeout_ms):
        if not self.pending:
            raise TimeoutError
        return self.pending.pop(0)

    def nvmlDeviceGetTotalEccErrors(self, h, kind, counter):
        return self.ecc[h[1]]

    def nvmlDeviceGetClockInfo(self, h, which):
        return 1965

    def nvmlDeviceGetTemperature(self, h, which):
        return 55

    def nvmlDeviceGetCurrentClocksThrottleReasons(self, h):
        return 4


def test_nvml_probe_reports_fatal_xids_and_new_ecc_errors():
    nv = FakeNVML()
    probe = NVMLProbe(nvml=nv)
    assert probe.available and probe.poll() == []
    nv.pending = [FakeEvent(("h", 1), 79), FakeEvent(("h", 0), 13)]
    nv.ecc[0] = 2
    evs = probe.poll()
    assert [(e.device, e.kind, e.fatal) for e in evs] == [("cuda:1", "xid", True), ("cuda:0", "xid", False),
                                                         ("cuda:0", "ecc", True)]
    assert evs[0].matches("cuda:1") and not evs[0].matches("cuda:0")
    assert probe.poll() == [], "an unchanged ECC count is not a new event"
    assert probe.throttle(0) == {"sm_clock": 1965, "temp": 55, "throttle": 4}
    assert 79 in FATAL_XIDS and 13 not in FATAL_XIDS


def test_nvml_probe_is_a_noop_without_nvml():
    class Broken:
        def nvmlInit(self):
            raise OSError("no driver")

    probe = NVMLProbe(nvml=Broken())
    assert not probe.available and probe.poll() == [] and probe.throttle(0) == {}


def test_ib_port_probe_on_a_fake_sysfs(tmp_path):
    for hca, state in (("mlx5_0", "4: ACTIVE"), ("mlx5_1", "1: DOWN")):
        d = tmp_path / hca / "ports" / "1"
        d.mkdir(parents=True)
        (d / "state").write_text(state + "\n")
    evs = IBPortProbe(str(tmp_path)).poll()
    assert len(evs) == 1 and not evs[0].fatal and "mlx5_1" in evs[0].detail
    (tmp_path / "mlx5_0" / "ports" / "1" / "state").write_text("1: DOWN\n")
    evs = CompositeProbe(IBPortProbe(str(tmp_path)), IBPortProbe(str(tmp_path / "missing"))).poll()
    assert len(evs) == 2 and all(e.fatal for e in evs)


def test_fault_grammar_round_trip_and_errors():
    spec = "kill@target=n0g3:iter=3:phase=forward;slow@target=n1g0:iter=5:factor=2.5:duration=30;" \
           "slow_link@target=n0:time=12.5:peer=10.0.0.2"
    faults = parse_faults(spec)
    assert [f.kind for f in faults] == [FaultKind.KILL, FaultKind.SLOW_COMPUTE, FaultKind.SLOW_LINK]
    assert faults[1].factor == 2.5 and faults[1].duration == 30 and faults[2].param("peer") == "10.0.0.2"
    assert parse_faults(";".join(f.to_spec() for f in faults)) == faults
    for bad in ("kill", "kill@iter=3", "kill@target=a:oops", "melt@target=a"):
        with pytest.raises(ValueError):
            parse_faults(bad)


def test_in_process_injector_padding_and_link_delay():
    faults = parse_faults("slow@target=w1:iter=2:factor=3;slow_link@target=w1:iter=0:delay_s=0.04:peer=w2")
    inj = FaultInjector("w1", faults)
    assert inj.compute_factor() == 1.0
    inj.on_hook(2, "forward")
    assert inj.compute_factor() == 3.0
    assert inj.link_delay("w2") == pytest.approx(0.04) and inj.link_delay("w3") == 0.0
    other = FaultInjector("w0", faults)
    other.on_hook(9, "forward")
    assert other.compute_factor() == 1.0, "faults only fire on their target"


def test_external_injector_dry_run_gate_and_schedule():
    faults = parse_faults("hang@target=n0g1:time=1:duration=2:pid=4242;power_cap@target=n0:time=0.5:watts=600")
    dry = ExternalInjector()
    log = run_schedule(faults, dry, clock=lambda: 0.0, sleep=lambda s: None)
    assert [(t, a) for t, _, a in log] == [(0.5, "apply"), (1.0, "apply"), (3.0, "revert")]
    assert dry.executed == [["nvidia-smi", "-i", "0", "-pl", "600"], ["kill", "-STOP", "4242"],
                            ["kill", "-CONT", "4242"]]
    ran = []
    live = ExternalInjector(dry_run=False, runner=lambda argv: ran.append(argv) or 0)
    with pytest.raises(PermissionError):
        live.apply(faults[1])  # changes a GPU setting: refused unless explicitly allowed
    live.apply(faults[0])
    assert ran == [["kill", "-STOP", "4242"]]


def test_intervals():
    assert iv.even_split(10, 3) == [(0, 4), (4, 7), (7, 10)]
    assert iv.is_partition(iv.even_split(7, 7), 7)
    assert iv.intersect((0, 5), (3, 9)) == (3, 5) and iv.intersect((0, 3), (3, 9)) is None
    assert iv.refine([iv.even_split(12, 4), iv.even_split(12, 3)]) == [(0, 3), (3, 4), (4, 6), (6, 8), (8, 9),
                                                                        (9, 12)]
    assert iv.overlaps([(0, 6), (6, 12)], [(0, 4), (4, 8), (8, 12)]) == [
        (0, 0, (0, 4)), (0, 1, (4, 6)), (1, 1, (6, 8)), (1, 2, (8, 12))]
    assert iv.locate(iv.even_split(12, 3), (5, 7)) == 1
    with pytest.raises(ValueError):
        iv.even_split(3, 0)


def test_group_specs_layers_and_order():
    specs = [GroupSpec("tp/r0/s0", (0, 1), "tp"), GroupSpec("tp/r0/s1", (2, 3), "tp"),
             GroupSpec("dp/a", (0, 2), "dp"), GroupSpec("dp/b", (1, 3), "dp"), GroupSpec("solo", (4,), "tp"),
             GroupSpec("dup", (0, 1), "x")]
    layers = split_layers(specs)
    for layer in layers:
        ranks = [r for s in layer for r in s.ranks]
        assert len(ranks) == len(set(ranks))
    names = {s.name for layer in layers for s in layer}
    assert "solo" not in names and len({s.ranks for layer in layers for s in layer}) == 4
    assert [s.name for s in canonical_order(specs)][:2] == ["dp/a", "dp/b"]
    with pytest.raises(ValueError):
        GroupSpec("bad", (1, 0))
    assert GroupSpec("keep", (5,), keep_singleton=True).materialized


def test_generation_hooks_order_and_graph_recapture():
    calls = []

    class Rec:
        def __init__(self, name):
            self.name = name

        def teardown(self):
            calls.append(("teardown", self.name))
            if self.name == "bad":
                raise RuntimeError("boom")

        def rebuild(self, comms, payload):
            calls.append(("rebuild", self.name))

    class Engine:
        def __init__(self):
            self.graphs = 0

        def drop_graphs(self):
            calls.append(("drop",))
            self.graphs = 0

        def capture_graphs(self):
            calls.append(("capture",))
            self.graphs += 1

    eng = Engine()
    heaps = []
    heap_hook = SymmetricHeapHook(lambda comms, payload: heaps.append(payload["gen"]) or type(
        "Heap", (), {"close": lambda self: calls.append(("close-heap",))})())
    graph = CudaGraphHook(lambda: eng, warmup=2)
    hooks = GenerationHooks([Rec("a"), heap_hook, Rec("bad"), graph])
    hooks.rebuild(None, {"gen": 1})
    errors = hooks.teardown()
    assert errors and "boom" in errors[0]
    # teardown runs in reverse registration order and survives a failing hook
    assert calls[:2] == [("rebuild", "a"), ("rebuild", "bad")]
    assert calls[2:] == [("drop",), ("teardown", "bad"), ("close-heap",), ("teardown", "a")]
    calls.clear()
    hooks.rebuild(None, {"gen": 2})
    hooks.after_iteration(0)
    assert ("capture",) not in calls
    hooks.after_iteration(1)
    hooks.after_iteration(2)
    assert calls.count(("capture",)) == 1 and graph.captures == 1 and heaps == [1, 2]
    assert heap_hook.rebuilds == 2
