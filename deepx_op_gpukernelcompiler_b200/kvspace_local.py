"""In-process stand-in for the external ``kvspace`` client.

The reference reads kvlang programs from kvspace, an external key/value
server, through ``from kvspace import KVSpace, ErrNotFound, connect``
(deepx_op_gpukernelcompiler/kvfunc.py:10, workflow.py:11).  Neither that
client nor its server ships with the reference, so this module provides the
surface the reference uses, backed by a dict:

* ``KVSpace.get(key)`` -> value object with ``.kind`` and ``.as_str()``
  (kvfunc.py:18,48,57-58); raises ``ErrNotFound`` for a missing key;
* ``KVSpace.list(prefix)`` -> names of the direct children of ``prefix``
  (kvfunc.py:40); raises ``ErrNotFound`` when nothing lives under it;
* ``connect()`` -> a process-wide store (workflow.py:38).

When the real ``kvspace`` package is importable, ``connect()`` returns the
real client instead, so the same code talks to a live server.
"""
from __future__ import annotations

import threading


class ErrNotFound(KeyError):
    """Raised for a key (or prefix) with no value."""


class Value:
    """A stored value: ``kind`` is ``"string"`` for the slots kvlang writes."""

    __slots__ = ("kind", "_data")

    def __init__(self, data):
        self._data = data
        self.kind = "string" if isinstance(data, str) else type(data).__name__

    def as_str(self) -> str:
        if not isinstance(self._data, str):
            raise TypeError(f"value of kind {self.kind!r} is not a string")
        return self._data

    def __repr__(self) -> str:
        return f"Value({self._data!r})"


class KVSpace:
    """Dict-backed key/value space with '/'-separated hierarchical keys."""

    def __init__(self):
        self._data: dict[str, Value] = {}
        self._lock = threading.Lock()

    def set(self, key: str, value) -> None:
        with self._lock:
            self._data[key] = value if isinstance(value, Value) else Value(value)

    def get(self, key: str) -> Value:
        with self._lock:
            try:
                return self._data[key]
            except KeyError:
                raise ErrNotFound(key) from None

    def delete(self, key: str) -> None:
        with self._lock:
            self._data.pop(key, None)

    def list(self, prefix: str) -> list[str]:
        base = prefix.rstrip("/") + "/"
        with self._lock:
            children = {k[len(base):].split("/", 1)[0] for k in self._data if k.startswith(base)}
        if not children:
            raise ErrNotFound(prefix)
        return sorted(children)

    def keys(self) -> list[str]:
        with self._lock:
            return sorted(self._data)


_default: KVSpace | None = None
_default_lock = threading.Lock()


def local_space() -> KVSpace:
    """The process-wide in-memory space."""
    global _default
    with _default_lock:
        if _default is None:
            _default = KVSpace()
        return _default


def connect(use_real: bool = True):
    """A real kvspace client if the package is installed, else the local space."""
    if use_real:
        try:
            import kvspace  # type: ignore[import-not-found]
        except ImportError:
            pass
        else:
            return kvspace.connect()
    return local_space()


def not_found_errors() -> tuple[type[BaseException], ...]:
    """Exception types meaning "no such key": ours, plus the real client's."""
    errs: list[type[BaseException]] = [ErrNotFound]
    try:
        from kvspace import ErrNotFound as RealErrNotFound  # type: ignore[import-not-found]
    except ImportError:
        pass
    else:
        errs.append(RealErrNotFound)
    return tuple(errs)
