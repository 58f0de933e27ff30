"""Fault injection.

* ``FaultInjector`` runs inside a worker and fires at deterministic hook points
  ``(iteration >= iter, phase)`` with phases ``forward``, ``backward``, ``reduce``, ``step``,
  ``loss``: SIGKILL itself, SIGSTOP itself (optionally resumed by a SIGCONT timer), pad compute by
  busy-waiting (fail-slow), or delay a link.  All of it happens on the host: a killed or stopped
  process leaves between kernel launches, never in the middle of a GPU operation.
* ``ExternalInjector`` builds (and, when allowed, runs) host commands that emulate hardware
  faults on a cluster: kill / stop, NIC down, bandwidth contention, and -- only with
  ``allow_device_settings=True`` -- SM clock locks, power caps and DCGM XID injection.  It is a
  dry run by default; on shared GPUs the device-setting faults stay dry-run only.

Spec grammar (``RESIHP_FAULTS`` or ``parse_faults``), same as the reference
(``resihp/inject/faults.py:35-287``)::

    kind@key=value:key=value;kind@...      e.g.  kill@iter=5:target=n0g1;slow@iter=10:target=n1g0:factor=2
Reserved keys: target, iter, time, duration, factor, phase; the rest go to ``params``.
"""

from __future__ import annotations

import os
import shlex
import signal
import subprocess
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Callable

from ..utils.log import get_logger

log = get_logger(__name__)


class FaultKind(str, Enum):
    KILL = "kill"
    HANG = "hang"
    SLOW_COMPUTE = "slow"
    SLOW_LINK = "slow_link"
    XID = "xid"
    NIC_DOWN = "nic_down"
    POWER_CAP = "power_cap"


DEVICE_SETTING_KINDS = frozenset({FaultKind.XID, FaultKind.POWER_CAP})


@dataclass(frozen=True)
class FaultSpec:
    kind: FaultKind
    target: str
    at_iteration: int | None = None
    at_time: float | None = None
    duration: float | None = None
    factor: float = 1.0
    phase: str = "forward"
    params: tuple[tuple[str, str], ...] = field(default_factory=tuple)

    def param(self, key: str, default: str | None = None) -> str | None:
        return dict(self.params).get(key, default)

    def to_spec(self) -> str:
        kv = [f"target={self.target}"]
        if self.at_iteration is not None:
            kv.append(f"iter={self.at_iteration}")
        if self.at_time is not None:
            kv.append(f"time={self.at_time}")
        if self.duration is not None:
            kv.append(f"duration={self.duration}")
        if self.factor != 1.0:
            kv.append(f"factor={self.factor}")
        if self.phase != "forward":
            kv.append(f"phase={self.phase}")
        kv += [f"{k}={v}" for k, v in self.params]
        return f"{self.kind.value}@" + ":".join(kv)


_RESERVED = {"target", "iter", "time", "duration", "factor", "phase"}


def parse_faults(spec: str | None) -> list[FaultSpec]:
    if not spec:
        return []
    out = []
    for item in (s.strip() for s in spec.split(";")):
        if not item:
            continue
        kind, sep, rest = item.partition("@")
        if not sep:
            raise ValueError(f"fault {item!r} must look like kind@key=value:...")
        kv: dict[str, str] = {}
        for tok in rest.split(":"):
            if not tok:
                continue
            k, eq, v = tok.partition("=")
            if not eq:
                raise ValueError(f"bad token {tok!r} in fault {item!r}")
            kv[k.strip()] = v.strip()
        if "target" not in kv:
            raise ValueError(f"fault {item!r} has no target")
        out.append(FaultSpec(kind=FaultKind(kind.strip()), target=kv["target"],
                             at_iteration=int(kv["iter"]) if "iter" in kv else None,
                             at_time=float(kv["time"]) if "time" in kv else None,
                             duration=float(kv["duration"]) if "duration" in kv else None,
                             factor=float(kv.get("factor", 1.0)), phase=kv.get("phase", "forward"),
                             params=tuple(sorted((k, v) for k, v in kv.items() if k not in _RESERVED))))
    return out


class FaultInjector:
    def __init__(self, worker_id: str, faults: list[FaultSpec], *, start_time: float | None = None,
                 kill_fn: Callable[[], None] | None = None):
        self.worker_id = worker_id
        self.faults = [f for f in faults if f.target in (worker_id, "*")]
        self.fired: set[int] = set()
        self.start_time = time.monotonic() if start_time is None else start_time
        self._kill_fn = kill_fn
        self._slow_until: float | None = None
        self._slow_factor = 1.0
        self._link_delay: dict[str, float] = {}

    def on_hook(self, iteration: int, phase: str) -> None:
        now = time.monotonic()
        for i, f in enumerate(self.faults):
            if i in self.fired or (f.at_iteration is None and f.at_time is None):
                continue
            if f.at_iteration is not None and (iteration < f.at_iteration or phase != f.phase):
                continue
            if f.at_time is not None and now - self.start_time < f.at_time:
                continue
            self.fired.add(i)
            self._fire(f, now)

    def _fire(self, f: FaultSpec, now: float) -> None:
        log.warning("injecting %s on %s", f.to_spec(), self.worker_id)
        if f.kind == FaultKind.KILL:
            (self._kill_fn or (lambda: os.kill(os.getpid(), signal.SIGKILL)))()
        elif f.kind == FaultKind.HANG:
            if f.duration is not None:
                subprocess.Popen(["sh", "-c", f"sleep {f.duration}; kill -CONT {os.getpid()}"])
            os.kill(os.getpid(), signal.SIGSTOP)
        elif f.kind == FaultKind.SLOW_COMPUTE:
            self._slow_factor = max(1.0, f.factor)
            self._slow_until = None if f.duration is None else now + f.duration
        elif f.kind == FaultKind.SLOW_LINK:
            self._link_delay[f.param("peer", "*")] = float(f.param("delay_s", "0.01"))
        else:
            raise ValueError(f"{f.kind.value} cannot be injected in-process; use ExternalInjector")

    def compute_factor(self) -> float:
        if self._slow_until is not None and time.monotonic() > self._slow_until:
            self._slow_factor, self._slow_until = 1.0, None
        return self._slow_factor

    def pad_compute(self, elapsed_s: float) -> float:
        """Busy-wait so a chunk that took ``elapsed_s`` looks ``factor`` times slower."""
        factor = self.compute_factor()
        if factor <= 1.0 or elapsed_s <= 0:
            return 0.0
        pad = (factor - 1.0) * elapsed_s
        end = time.perf_counter() + pad
        while time.perf_counter() < end:
            pass
        return pad

    def link_delay(self, peer: str) -> float:
        d = self._link_delay.get(peer, self._link_delay.get("*", 0.0))
        if d > 0:
            time.sleep(d)
        return d


_INJECTOR: FaultInjector | None = None


def get_injector() -> FaultInjector:
    """Process-wide injector from ``RESIHP_FAULTS`` and ``RESIHP_WORKER_ID``."""
    global _INJECTOR
    if _INJECTOR is None:
        _INJECTOR = FaultInjector(os.environ.get("RESIHP_WORKER_ID", ""), parse_faults(os.environ.get("RESIHP_FAULTS")))
    return _INJECTOR


def reset_injector(injector: FaultInjector | None = None) -> None:
    global _INJECTOR
    _INJECTOR = injector


@dataclass
class ExternalCommand:
    apply: list[str]
    revert: list[str] | None = None


class ExternalInjector:
    """Host-level fault emulation; dry run unless ``dry_run=False``.  Commands that change a
    GPU's settings (clock lock, power cap, XID injection) additionally need
    ``allow_device_settings=True`` and are refused otherwise."""

    def __init__(self, dry_run: bool = True, runner: Callable[[list[str]], int] | None = None,
                 allow_device_settings: bool = False):
        self.dry_run = dry_run
        self.allow_device_settings = allow_device_settings
        self.executed: list[list[str]] = []
        self._runner = runner or (lambda cmd: subprocess.call(cmd))

    @staticmethod
    def commands(f: FaultSpec) -> ExternalCommand:
        gpu = f.param("gpu", "0")
        if f.kind == FaultKind.KILL:
            return ExternalCommand(["kill", "-9", f.param("pid", "0")])
        if f.kind == FaultKind.HANG:
            pid = f.param("pid", "0")
            return ExternalCommand(["kill", "-STOP", pid], ["kill", "-CONT", pid])
        if f.kind == FaultKind.SLOW_COMPUTE:
            base = float(f.param("base_mhz", "1965"))
            mhz = str(int(base / max(f.factor, 1.0)))
            return ExternalCommand(["nvidia-smi", "-i", gpu, "-lgc", f"{mhz},{mhz}"], ["nvidia-smi", "-i", gpu, "-rgc"])
        if f.kind == FaultKind.POWER_CAP:
            return ExternalCommand(["nvidia-smi", "-i", gpu, "-pl", f.param("watts", "500")],
                                   ["nvidia-smi", "-i", gpu, "-pl", f.param("default_watts", "1000")])
        if f.kind == FaultKind.XID:
            # DCGM field 230 (XID errors): exercises the health-monitor path
            return ExternalCommand(["dcgmi", "test", "--inject", "--gpuid", gpu, "-f", "230", "-v",
                                    f.param("xid", "79")])
        if f.kind == FaultKind.NIC_DOWN:
            iface = f.param("iface", "ib0")
            return ExternalCommand(["ip", "link", "set", "dev", iface, "down"], ["ip", "link", "set", "dev", iface, "up"])
        if f.kind == FaultKind.SLOW_LINK:
            return ExternalCommand(["python", "-m", "resihp_megatron_b200.inject.contention", "--host",
                                    f.param("peer", "127.0.0.1"), "--port", f.param("port", "29700"), "--seconds",
                                    str(f.duration or 60)])
        raise ValueError(f"unsupported external fault {f.kind}")

    @staticmethod
    def changes_device_settings(f: FaultSpec) -> bool:
        return f.kind in DEVICE_SETTING_KINDS or f.kind == FaultKind.SLOW_COMPUTE

    def apply(self, f: FaultSpec) -> ExternalCommand:
        cmd = self.commands(f)
        self._run(cmd.apply, f)
        return cmd

    def revert(self, f: FaultSpec) -> None:
        cmd = self.commands(f)
        if cmd.revert:
            self._run(cmd.revert, f)

    def _run(self, argv: list[str], f: FaultSpec) -> None:
        self.executed.append(argv)
        if self.dry_run:
            log.warning("[dry-run] %s", shlex.join(argv))
            return
        if self.changes_device_settings(f) and not self.allow_device_settings:
            raise PermissionError(f"{f.kind.value} changes GPU settings; pass allow_device_settings=True")
        rc = self._runner(argv)
        if rc != 0:
            raise RuntimeError(f"fault command failed ({rc}): {shlex.join(argv)}")


def run_schedule(faults: list[FaultSpec], injector: ExternalInjector, *, clock: Callable[[], float] = time.monotonic,
                 sleep: Callable[[float], None] = time.sleep) -> list[tuple[float, FaultSpec, str]]:
    """Run time-triggered faults and their reverts in time order; returns the event log."""
    t0 = clock()
    events: list[tuple[float, str, FaultSpec]] = []
    for f in faults:
        if f.at_time is None:
            continue
        events.append((f.at_time, "apply", f))
        if f.duration is not None:
            events.append((f.at_time + f.duration, "revert", f))
    events.sort(key=lambda e: (e[0], e[1] != "revert"))
    log_ = []
    for at, action, f in events:
        wait = at - (clock() - t0)
        if wait > 0:
            sleep(wait)
        (injector.apply if action == "apply" else injector.revert)(f)
        log_.append((at, f, action))
    return log_
