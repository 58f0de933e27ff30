"""Key-value store for control state: generation, membership, plans and the leader lease.

``KVStore`` is the protocol; ``InMemoryKV`` backs tests and single-coordinator jobs (with an
injectable clock for lease tests); ``EtcdKV`` is the production backend that makes the
coordinator replaceable.  ``put_if`` is the fenced write: it succeeds only while the guard
key (the leader key) still names this coordinator (reference: ``resihp/control/kvstore.py``).
Keys used by the coordinator: ``{ns}/leader``, ``{ns}/state``, ``{ns}/plan/{gen}``.
"""

from __future__ import annotations

import itertools
import threading
import time
from typing import Callable, Protocol


class KVStore(Protocol):
    def get(self, key: str) -> str | None: ...
    def get_prefix(self, prefix: str) -> dict[str, str]: ...
    def put(self, key: str, value: str, lease: int | None = None) -> None: ...
    def cas(self, key: str, expected: str | None, value: str, lease: int | None = None) -> bool: ...
    def put_if(self, key: str, value: str, guard_key: str, guard_value: str) -> bool: ...
    def delete(self, key: str) -> None: ...
    def grant_lease(self, ttl: float) -> int: ...
    def keepalive(self, lease: int) -> bool: ...
    def revoke(self, lease: int) -> None: ...


class InMemoryKV:
    """Thread-safe dict with leases; a key bound to an expired lease disappears."""

    def __init__(self, clock: Callable[[], float] = time.monotonic):
        self._clock = clock
        self._mu = threading.RLock()
        self._kv: dict[str, str] = {}
        self._owner: dict[str, int] = {}          # key -> lease id
        self._deadline: dict[int, float] = {}     # lease -> expiry time
        self._ttl: dict[int, float] = {}
        self._next = itertools.count(1)

    def _gc(self) -> None:
        now = self._clock()
        expired = [l for l, t in self._deadline.items() if t <= now]
        for l in expired:
            del self._deadline[l]
            self._ttl.pop(l, None)
        if expired:
            gone = set(expired)
            for k in [k for k, l in self._owner.items() if l in gone]:
                self._kv.pop(k, None)
                del self._owner[k]

    def _set(self, key: str, value: str, lease: int | None) -> None:
        if lease is not None and lease not in self._deadline:
            raise KeyError(f"lease {lease} expired")
        self._kv[key] = value
        if lease is None:
            self._owner.pop(key, None)
        else:
            self._owner[key] = lease

    def get(self, key: str) -> str | None:
        with self._mu:
            self._gc()
            return self._kv.get(key)

    def get_prefix(self, prefix: str) -> dict[str, str]:
        with self._mu:
            self._gc()
            return {k: v for k, v in self._kv.items() if k.startswith(prefix)}

    def put(self, key: str, value: str, lease: int | None = None) -> None:
        with self._mu:
            self._gc()
            self._set(key, value, lease)

    def cas(self, key: str, expected: str | None, value: str, lease: int | None = None) -> bool:
        with self._mu:
            self._gc()
            if self._kv.get(key) != expected:
                return False
            self._set(key, value, lease)
            return True

    def put_if(self, key: str, value: str, guard_key: str, guard_value: str) -> bool:
        with self._mu:
            self._gc()
            if self._kv.get(guard_key) != guard_value:
                return False
            self._set(key, value, None)
            return True

    def delete(self, key: str) -> None:
        with self._mu:
            self._kv.pop(key, None)
            self._owner.pop(key, None)

    def grant_lease(self, ttl: float) -> int:
        with self._mu:
            lid = next(self._next)
            self._deadline[lid] = self._clock() + ttl
            self._ttl[lid] = ttl
            return lid

    def keepalive(self, lease: int) -> bool:
        with self._mu:
            self._gc()
            if lease not in self._deadline:
                return False
            self._deadline[lease] = self._clock() + self._ttl[lease]
            return True

    def revoke(self, lease: int) -> None:
        with self._mu:
            if lease in self._deadline:
                self._deadline[lease] = float("-inf")
            self._gc()


class EtcdKV:
    """etcd v3 backend; needs the optional ``etcd3`` package."""

    def __init__(self, host: str = "127.0.0.1", port: int = 2379, **kwargs):
        try:
            import etcd3  # type: ignore
        except ImportError as e:  # pragma: no cover - not installed in CI
            raise RuntimeError("EtcdKV needs the 'etcd3' package") from e
        self._c = etcd3.client(host=host, port=port, **kwargs)
        self._leases: dict[int, object] = {}

    def _lease(self, lease):
        return self._leases.get(lease) if lease else None

    def get(self, key):
        v, _ = self._c.get(key)
        return None if v is None else v.decode()

    def get_prefix(self, prefix):
        return {meta.key.decode(): v.decode() for v, meta in self._c.get_prefix(prefix)}

    def put(self, key, value, lease=None):
        self._c.put(key, value, lease=self._lease(lease))

    def cas(self, key, expected, value, lease=None):
        tx = self._c.transactions
        cond = tx.version(key) == 0 if expected is None else tx.value(key) == expected
        ok, _ = self._c.transaction(compare=[cond], success=[tx.put(key, value, lease=self._lease(lease))],
                                    failure=[])
        return ok

    def put_if(self, key, value, guard_key, guard_value):
        tx = self._c.transactions
        ok, _ = self._c.transaction(compare=[tx.value(guard_key) == guard_value],
                                    success=[tx.put(key, value)], failure=[])
        return ok

    def delete(self, key):
        self._c.delete(key)

    def grant_lease(self, ttl):
        lease = self._c.lease(max(1, int(round(ttl))))
        self._leases[lease.id] = lease
        return lease.id

    def keepalive(self, lease):
        obj = self._leases.get(lease)
        if obj is None:
            return False
        try:
            r = list(obj.refresh())
            return bool(r) and r[0].TTL > 0
        except Exception:  # noqa: BLE001 - any etcd error means the lease is gone
            return False

    def revoke(self, lease):
        obj = self._leases.pop(lease, None)
        if obj is not None:
            obj.revoke()
