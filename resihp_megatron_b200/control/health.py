"""Node health probes: NVML (critical XID events, uncorrected ECC errors, and clock / throttle
readings as side information) and InfiniBand port state from sysfs.

A probe whose facility is missing reports nothing, so the same agent runs on a CPU-only host.
``NVMLProbe`` accepts an ``nvml`` module object, which lets tests drive it with a fake.  The
probes only read device state; nothing here changes a GPU setting.
Parity: ``resihp/control/health.py:13-120`` (the fatal XID set is the same operational list).
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass
from pathlib import Path

# XIDs after which the GPU is lost for this job
FATAL_XIDS = frozenset({48, 61, 62, 63, 64, 74, 79, 92, 94, 95, 119, 120, 140})


@dataclass(frozen=True)
class HealthEvent:
    device: str          # "cuda:<i>", or "*" for the whole node
    kind: str            # xid | ecc | ib_port
    fatal: bool
    detail: str = ""

    def matches(self, worker_device: str) -> bool:
        return self.device in ("*", worker_device)

    def describe(self) -> str:
        return f"{self.kind} on {self.device}: {self.detail}"


class NVMLProbe:
    """Critical XIDs (drained from an NVML event set) and growth of the uncorrected ECC count."""

    def __init__(self, nvml=None, device_indices: list[int] | None = None):
        self.nvml = nvml
        self._handles: dict[int, object] = {}
        self._event_set = None
        self._ecc_seen: dict[int, int] = {}
        self._ok = self._open(device_indices)

    def _open(self, device_indices) -> bool:
        try:
            if self.nvml is None:
                import pynvml  # nvidia-ml-py

                self.nvml = pynvml
            nv = self.nvml
            nv.nvmlInit()
            wanted = range(nv.nvmlDeviceGetCount()) if device_indices is None else device_indices
            self._handles = {i: nv.nvmlDeviceGetHandleByIndex(i) for i in wanted}
            self._event_set = nv.nvmlEventSetCreate()
            for handle in self._handles.values():
                with contextlib.suppress(Exception):  # some SKUs do not deliver XID events
                    nv.nvmlDeviceRegisterEvents(handle, nv.nvmlEventTypeXidCriticalError, self._event_set)
            return True
        except Exception:  # noqa: BLE001 -- no NVML on this host
            return False

    @property
    def available(self) -> bool:
        return self._ok

    def _device_name(self, handle) -> str:
        found = [i for i, h in self._handles.items() if h == handle]
        return f"cuda:{found[0]}" if found else "*"

    def _xid_events(self) -> list[HealthEvent]:
        out = []
        while True:
            try:
                ev = self.nvml.nvmlEventSetWait(self._event_set, 0)
            except Exception:  # noqa: BLE001 -- nothing pending
                return out
            xid = int(ev.eventData)
            out.append(HealthEvent(self._device_name(ev.device), "xid", xid in FATAL_XIDS, f"XID {xid}"))

    def _ecc_events(self) -> list[HealthEvent]:
        nv, out = self.nvml, []
        for i, handle in self._handles.items():
            try:
                count = nv.nvmlDeviceGetTotalEccErrors(handle, nv.NVML_MEMORY_ERROR_TYPE_UNCORRECTED,
                                                       nv.NVML_VOLATILE_ECC)
            except Exception:  # noqa: BLE001
                continue
            before = self._ecc_seen.setdefault(i, count)
            if count > before:
                out.append(HealthEvent(f"cuda:{i}", "ecc", True, f"uncorrected ECC count {count}"))
            self._ecc_seen[i] = count
        return out

    def poll(self) -> list[HealthEvent]:
        return self._xid_events() + self._ecc_events() if self._ok else []

    def throttle(self, index: int) -> dict:
        """SM clock, temperature and throttle reasons: side information for the fail-slow
        detector, never a trigger by themselves."""
        handle = self._handles.get(index) if self._ok else None
        if handle is None:
            return {}
        nv = self.nvml
        readers = {"sm_clock": lambda: nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM),
                   "temp": lambda: nv.nvmlDeviceGetTemperature(handle, nv.NVML_TEMPERATURE_GPU),
                   "throttle": lambda: nv.nvmlDeviceGetCurrentClocksThrottleReasons(handle)}
        readings = {}
        for name, read in readers.items():
            with contextlib.suppress(Exception):
                readings[name] = read()
        return readings


class IBPortProbe:
    """A port not ACTIVE degrades the node (a fail-slow candidate); all ports down isolate it."""

    def __init__(self, root: str = "/sys/class/infiniband"):
        self.root = Path(root)

    def poll(self) -> list[HealthEvent]:
        if not self.root.is_dir():
            return []
        ports = sorted(self.root.glob("*/ports/*/state"))
        down = []
        for path in ports:
            state = path.read_text().strip()
            if "ACTIVE" in state:
                continue
            hca, port = path.parts[-4], path.parts[-2]
            down.append(f"{hca} port {port} {state}")
        isolated = len(down) == len(ports) > 0
        return [HealthEvent("*", "ib_port", isolated, what) for what in down]


class CompositeProbe:
    def __init__(self, *probes):
        self.probes = probes

    def poll(self) -> list[HealthEvent]:
        return [ev for probe in self.probes for ev in probe.poll()]
