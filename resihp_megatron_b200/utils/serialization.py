"""Canonical JSON for plans, IR, payloads and control messages.

``dumps`` is deterministic -- keys sorted, no whitespace, sets sorted, dataclasses and enums
lowered to plain values -- so every rank that serialises the same plan produces the same
bytes (and the same hash).  ``tuplify`` turns the lists of a decoded document back into
tuples, which is how plans hold their sequences.
Parity: ``resihp/utils/serialization.py:25-39`` (same canonical form).
"""

from __future__ import annotations

import dataclasses
import json
from enum import Enum
from functools import singledispatch
from typing import Any


@singledispatch
def to_jsonable(obj: Any) -> Any:
    """Plain JSON values for enums, dataclass instances, sets and tuples (recursively)."""
    is_record = dataclasses.is_dataclass(obj) and not isinstance(obj, type)
    return {k: to_jsonable(v) for k, v in vars_of(obj).items()} if is_record else obj


def vars_of(record) -> dict:
    return {f.name: getattr(record, f.name) for f in dataclasses.fields(record)}


@to_jsonable.register
def _(obj: Enum) -> Any:
    return obj.value


@to_jsonable.register
def _(obj: dict) -> Any:
    return {str(key): to_jsonable(val) for key, val in obj.items()}


@to_jsonable.register(set)
@to_jsonable.register(frozenset)
def _(obj) -> Any:
    return sorted(map(to_jsonable, obj))


@to_jsonable.register(list)
@to_jsonable.register(tuple)
def _(obj) -> Any:
    return list(map(to_jsonable, obj))


_CANONICAL = json.JSONEncoder(sort_keys=True, separators=(",", ":"))


def dumps(obj: Any) -> str:
    return _CANONICAL.encode(to_jsonable(obj))


loads = json.loads


def tuplify(obj: Any) -> Any:
    """Lists become tuples, recursively (dict keys and scalars are kept)."""
    kind = type(obj)
    if kind is list:
        return tuple(tuplify(v) for v in obj)
    return {k: tuplify(v) for k, v in obj.items()} if kind is dict else obj
