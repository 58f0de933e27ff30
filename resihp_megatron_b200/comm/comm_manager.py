"""ResilientCommManager: generation-scoped communicators that are rebuilt without hanging.

Hang causes designed out:
* dead ranks taking part in group creation -> survivors-only creation: NCCL ``shrink_group``
  (with abort of whatever the dead ranks left in flight) when the new world is an
  order-preserving subset of the old one and NCCL >= 2.27.3, else a fresh world on a
  generation-scoped ``PrefixStore`` of the coordinator-hosted ``TCPStore``;
* creation order depending on local state -> plan-derived canonical order: one ``split_group``
  per layer of disjoint groups on NCCL, or ``new_group`` for every group on every rank in that
  order on gloo;
* a rendezvous store on a training rank -> the store lives on the coordinator;
* blocking forever in a collective -> ``guarded_wait`` (abortable, deadline) and a validation
  all-reduce of ones on every group under a deadline before the generation may report READY
  (failure raises ``GenerationBuildError`` naming the suspect ranks).

``abort()`` (called from the control-client thread) sets the abort flag, aborts every live NCCL
group and sets the device abort word that the package's peer-memory kernels poll, so survivors
leave in-flight fused kernels at once.  Gloo groups are aborted when their generation is torn
down: a gloo op that lost its peer stays in flight until its timeout, and destroying its group
would otherwise wait for it while the next generation's rendezvous runs out of time.  (Reference: ``resihp/comm/comm_manager.py:31-329``.)
"""

from __future__ import annotations

import datetime
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
import torch.distributed as dist
import torch.distributed.distributed_c10d as c10d

from .group_spec import GroupSpec, canonical_order, split_layers
from ..utils.log import get_logger

log = get_logger(__name__)


class CommAborted(RuntimeError):
    """The control plane aborted this generation's communicators."""


class CommTimeout(RuntimeError):
    """A guarded wait ran past its deadline."""


class GenerationBuildError(RuntimeError):
    def __init__(self, msg: str, suspects: tuple[int, ...] = ()):
        super().__init__(msg)
        self.suspects = suspects


@dataclass
class GenerationComms:
    generation: int
    rank: int
    world: tuple[str, ...]
    specs: dict[str, GroupSpec]
    groups: dict[str, Any]
    path: str
    build_seconds: float = 0.0
    stats: dict = field(default_factory=dict)

    @property
    def world_size(self) -> int:
        return len(self.world)

    def group(self, name: str):
        """Process group for ``name``; ``None`` if this rank is not a member or it has one rank."""
        if name not in self.specs:
            raise KeyError(f"unknown group {name}")
        return self.groups.get(name)

    def ranks(self, name: str) -> tuple[int, ...]:
        return self.specs[name].ranks

    def is_member(self, name: str) -> bool:
        return self.rank in self.specs[name].ranks

    def rank_of(self, worker_id: str) -> int:
        return self.world.index(worker_id)


def is_order_preserving_subset(new: list[str], old: tuple[str, ...]) -> bool:
    pos = {w: i for i, w in enumerate(old)}
    if any(w not in pos for w in new):
        return False
    idx = [pos[w] for w in new]
    return idx == sorted(idx)


class ResilientCommManager:
    def __init__(self, backend: str = "gloo", *, device: str | None = None, timeout_s: float = 60.0,
                 validate_timeout_s: float = 30.0, validate: bool = True, shrink: str = "auto",
                 subgroup_mode: str = "split", nccl_nonblocking: bool = True, poll_interval_s: float = 0.0005):
        if shrink not in ("auto", "never", "always"):
            raise ValueError(shrink)
        if subgroup_mode not in ("split", "local"):
            raise ValueError(subgroup_mode)
        self.backend = backend
        self.device = device
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.validate_timeout_s = validate_timeout_s
        self.validate = validate
        self.shrink = shrink
        self.subgroup_mode = subgroup_mode
        self.nccl_nonblocking = nccl_nonblocking
        self.poll_interval_s = poll_interval_s or 0.0005
        self.current: GenerationComms | None = None
        self._abort = threading.Event()
        self._lock = threading.Lock()
        self._live: list[Any] = []
        self._store_client = None
        self._store_addr: tuple[str, int] | None = None
        self._abort_hooks: list[Callable[[], None]] = []

    # ------------------------------------------------------------------ capabilities
    @staticmethod
    def capabilities() -> dict:
        caps = {"shrink_group": hasattr(dist, "shrink_group"), "split_group": hasattr(dist, "split_group"),
                "nccl": dist.is_nccl_available(), "gloo": dist.is_gloo_available(), "nccl_version": None}
        if torch.cuda.is_available() and dist.is_nccl_available():
            try:
                caps["nccl_version"] = torch.cuda.nccl.version()
            except Exception:  # noqa: BLE001
                pass
        return caps

    def can_shrink(self, new_world: list[str]) -> bool:
        if self.shrink == "never" or self.current is None or self.backend != "nccl":
            return False
        caps = self.capabilities()
        nccl_ok = caps["nccl_version"] is not None and tuple(caps["nccl_version"]) >= (2, 27, 3)
        if not (caps["shrink_group"] and nccl_ok and hasattr(c10d, "SHRINK_ABORT")):
            return False
        return len(new_world) < self.current.world_size and is_order_preserving_subset(new_world,
                                                                                       self.current.world)

    def add_abort_hook(self, fn: Callable[[], None]) -> None:
        """Extra action on abort (e.g. raising the device abort word of the symmetric heap)."""
        self._abort_hooks.append(fn)

    # ------------------------------------------------------------------ building
    def store_for(self, store_addr: tuple[str, int], prefix: str):
        if self._store_client is None or self._store_addr != tuple(store_addr):
            self._store_client = dist.TCPStore(store_addr[0], int(store_addr[1]), is_master=False,
                                               timeout=self.timeout, wait_for_workers=False)
            self._store_addr = tuple(store_addr)
        return dist.PrefixStore(prefix, self._store_client)

    def build(self, generation: int, world: list[str], my_id: str, specs: list[GroupSpec], *, store=None,
              store_addr: tuple[str, int] | None = None, store_prefix: str | None = None) -> GenerationComms:
        t0 = time.monotonic()
        self._abort.clear()
        rank = world.index(my_id)
        for s in specs:
            if any(r >= len(world) for r in s.ranks):
                raise ValueError(f"group {s.name} names a rank outside a world of {len(world)}")
        path = "shrink" if self.can_shrink(world) else "fresh"
        if self.shrink == "always" and path != "shrink":
            raise RuntimeError("shrink requested but this transition cannot shrink")
        if path == "shrink":
            keep = set(world)
            excluded = [i for i, w in enumerate(self.current.world) if w not in keep]
            dist.shrink_group(excluded, group=None, shrink_flags=c10d.SHRINK_ABORT)
        else:
            if store is None:
                if store_addr is None or store_prefix is None:
                    raise ValueError("a fresh world needs a store (or store_addr + store_prefix)")
                store = self.store_for(store_addr, store_prefix)
            self._teardown()
            self._init_world(rank, len(world), store)
        with self._lock:
            self._live = [c10d._get_default_group()]
        groups = self._make_subgroups(rank, specs)
        if self.validate:
            self._validate(len(world), groups, specs)
        comms = GenerationComms(generation, rank, tuple(world), {s.name: s for s in specs}, groups, path,
                                time.monotonic() - t0)
        self.current = comms
        log.info("generation %d built (%s) in %.3fs with %d groups", generation, path, comms.build_seconds,
                 len(groups))
        return comms

    def adopt(self, generation: int, world: list[str], my_id: str, specs: list[GroupSpec]) -> GenerationComms:
        """Use the already initialised default process group (a launcher's environment, e.g.
        ``torchrun``) as this generation's world and create the plan's subgroups on it."""
        t0 = time.monotonic()
        self._abort.clear()
        rank = world.index(my_id)
        if not dist.is_initialized() or dist.get_world_size() != len(world) or dist.get_rank() != rank:
            raise RuntimeError("adopt() needs an initialised default group matching the world")
        with self._lock:
            self._live = [c10d._get_default_group()]
        groups = self._make_subgroups(rank, specs)
        if self.validate:
            self._validate(len(world), groups, specs)
        comms = GenerationComms(generation, rank, tuple(world), {s.name: s for s in specs}, groups, "adopted",
                                time.monotonic() - t0)
        self.current = comms
        return comms

    def _init_world(self, rank: int, world_size: int, store) -> None:
        kw: dict = {"backend": self.backend, "store": store, "rank": rank, "world_size": world_size,
                    "timeout": self.timeout}
        if self.backend == "nccl":
            if self.device is not None:
                kw["device_id"] = torch.device(self.device)
            if self.nccl_nonblocking:
                opts = dist.ProcessGroupNCCL.Options()
                opts.config.blocking = 0
                kw["pg_options"] = opts
        dist.init_process_group(**kw)

    def _make_subgroups(self, rank: int, specs: list[GroupSpec]) -> dict[str, Any]:
        by_ranks: dict[tuple[int, ...], Any] = {}
        # split_group needs a device bound to the default group (NCCL with device_id); gloo
        # worlds use canonical-order new_group instead
        use_split = self.subgroup_mode == "split" and self.backend == "nccl" and self.device is not None
        if use_split:
            for layer in split_layers(specs):
                self._check_abort()
                pg = dist.split_group(split_ranks=[list(s.ranks) for s in layer], timeout=self.timeout,
                                      group_desc=f"resihp:{layer[0].kind}:{len(layer)}")
                for s in layer:
                    if rank in s.ranks:
                        by_ranks[s.ranks] = pg
        else:
            # every rank creates every group in the same canonical order (non-members too), so
            # c10d derives identical group names everywhere and creation cannot deadlock
            made: set[tuple[int, ...]] = set()
            for s in canonical_order(specs):
                if not s.materialized or s.ranks in made:
                    continue
                made.add(s.ranks)
                self._check_abort()
                pg = dist.new_group(list(s.ranks), timeout=self.timeout, group_desc=f"resihp:{s.name}")
                if rank in s.ranks:
                    by_ranks[s.ranks] = pg
        groups = {s.name: (by_ranks.get(s.ranks) if rank in s.ranks and s.materialized else None) for s in specs}
        with self._lock:
            self._live.extend(pg for pg in by_ranks.values() if pg not in self._live)
        return groups

    def _validate(self, world_size: int, groups: dict[str, Any], specs: list[GroupSpec]) -> None:
        dev = torch.device(self.device) if (self.backend == "nccl" and self.device) else torch.device("cpu")
        seen: set[int] = set()
        targets = [(c10d._get_default_group(), tuple(range(world_size)), "world")]
        targets += [(groups[s.name], s.ranks, s.name) for s in canonical_order(specs) if groups.get(s.name) is not None]
        for pg, ranks, name in targets:
            if id(pg) in seen:
                continue
            seen.add(id(pg))
            t = torch.ones(1, device=dev)
            try:
                self.guarded_wait(dist.all_reduce(t, group=pg, async_op=True), timeout=self.validate_timeout_s,
                                  what=f"validate {name}")
            except CommAborted:
                raise
            except (CommTimeout, RuntimeError) as e:
                raise GenerationBuildError(f"group {name} failed validation: {e}", suspects=tuple(ranks)) from e
            if int(t.item()) != pg.size():
                raise GenerationBuildError(f"group {name}: validation sum {t.item()} != {pg.size()}", tuple(ranks))

    # ------------------------------------------------------------------ waiting / aborting
    def _check_abort(self) -> None:
        if self._abort.is_set():
            raise CommAborted("communicators aborted by the control plane")

    def guarded_wait(self, work, timeout: float | None = None, what: str = "collective") -> None:
        """Wait for ``work`` while honouring aborts and a deadline.  Gloo cannot interrupt an
        in-flight op, so its blocking wait runs on a helper thread while this thread polls; on
        NCCL ``wait()`` only orders streams and hangs are broken by ``abort()``."""
        if self.backend == "nccl":
            self._check_abort()
            work.wait()
            return
        if work.is_completed():
            work.wait()
            return
        done = threading.Event()
        failure: list[BaseException] = []

        def waiter() -> None:
            try:
                work.wait()
            except BaseException as e:  # noqa: BLE001 - re-raised on the caller's thread
                failure.append(e)
            finally:
                done.set()

        threading.Thread(target=waiter, name="guarded-wait", daemon=True).start()
        deadline = None if timeout is None else time.monotonic() + timeout
        while not done.wait(self.poll_interval_s):
            if self._abort.is_set():
                raise CommAborted(f"{what} aborted by the control plane")
            if deadline is not None and time.monotonic() > deadline:
                raise CommTimeout(f"{what} timed out after {timeout}s")
        if failure:
            raise failure[0]

    def abort(self) -> None:
        """Thread safe; called from the control-client thread on RECONFIG_NOTICE."""
        self._abort.set()
        for fn in self._abort_hooks:
            try:
                fn()
            except Exception:  # noqa: BLE001 - best effort
                log.exception("abort hook raised")
        if self.backend != "nccl":
            return
        with self._lock:
            live = list(self._live)
        for pg in live:
            try:
                pg.abort()
            except Exception:  # noqa: BLE001 - the NCCL watchdog is the backstop
                pass

    @property
    def aborted(self) -> bool:
        return self._abort.is_set()

    def _teardown(self) -> None:
        if not dist.is_initialized():
            self.current = None
            return
        try:
            if self.backend == "nccl":
                c10d._abort_process_group(None)
            else:
                # a gloo op that lost its peer stays in flight until its timeout, and destroying
                # its group would wait for it: abort the groups first (returns at once)
                with self._lock:
                    live = list(self._live)
                for pg in live:
                    try:
                        pg.abort()
                    except Exception:  # noqa: BLE001 - older gloo builds: fall back to the wait
                        pass
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            log.exception("teardown of the previous generation failed; continuing")
        with self._lock:
            self._live = []
        self.current = None

    def destroy(self) -> None:
        self._teardown()
