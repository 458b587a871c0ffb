"""Cross-request state cache with the reference's API and eviction rules.

Same surface and semantics as d3trt/model/cache.py:24-184: ``tensor_bytes``,
``StateEntry``, and ``StateCache(capacity_bytes)`` — a byte-budgeted LRU of
state snapshots with ``get`` / ``put`` / ``acquire`` / ``release`` / ``drop`` /
``clear`` / ``get_or_compute`` / ``stats``; entries pinned by ``acquire`` are not
evicted, and eviction stops at the first pinned entry (the cache may then
overshoot until the batch releases it, cache.py:160-170).

With ``arena=SnapshotArena(...)`` a stored snapshot is packed into one block of
device memory (``pack_snapshot``: one copy launch) so the cache holds exactly
the bytes it counts, instead of the caller's tensors and whatever larger
buffers they are views of. Which entries are evicted is decided before the
copy and is the same set the reference evicts after inserting. If the arena
has no free range for the block (fragmentation), the entry keeps the caller's
tensors, as the reference does, and ``stats()["arena_fallbacks"]`` counts it.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Callable

from .snapshot import PackedSnapshot, SnapshotArena, SnapshotLayout, pack_snapshot


class StateCacheError(RuntimeError):
    """A cached state is missing, evicted while in use, or inconsistent."""


def tensor_bytes(obj: Any) -> int:
    """Bytes a tensor, a (nested) list/tuple of tensors or a dataclass reports (cache.py:24-34)."""
    if hasattr(obj, "numel") and hasattr(obj, "element_size"):
        return int(obj.numel()) * int(obj.element_size())
    if isinstance(obj, (list, tuple)):
        return sum(tensor_bytes(x) for x in obj)
    if hasattr(obj, "__dict__"):
        return sum(tensor_bytes(v) for v in vars(obj).values())
    if hasattr(obj, "__slots__"):
        return sum(tensor_bytes(getattr(obj, s)) for s in obj.__slots__ if hasattr(obj, s))
    return 0


@dataclass
class StateEntry:
    key: str
    snapshot: Any
    state_len: int
    nbytes: int
    media_hash: str = ""
    created: float = field(default_factory=time.monotonic)
    last_used: float = field(default_factory=time.monotonic)
    refcount: int = 0
    hits: int = 0


class StateCache:
    """A byte-budgeted LRU cache of state snapshots, optionally packed into an HBM arena."""

    def __init__(self, capacity_bytes: int, *, arena: SnapshotArena | None = None):
        if capacity_bytes < 0:
            raise ValueError("capacity_bytes must be >= 0")
        self.capacity_bytes = int(capacity_bytes)
        self.arena = arena
        self._entries: OrderedDict[str, StateEntry] = OrderedDict()
        self._bytes = 0
        self._lock = threading.RLock()
        self.hits = 0
        self.misses = 0
        self.evictions = 0
        self.rejected = 0
        self.arena_fallbacks = 0

    @property
    def bytes(self) -> int:
        return self._bytes

    @property
    def count(self) -> int:
        return len(self._entries)

    def __contains__(self, key: str) -> bool:
        with self._lock:
            return key in self._entries

    def stats(self) -> dict[str, Any]:
        with self._lock:
            total = self.hits + self.misses
            out = {
                "entries": len(self._entries),
                "bytes": self._bytes,
                "capacity_bytes": self.capacity_bytes,
                "hits": self.hits,
                "misses": self.misses,
                "hit_rate": round(self.hits / total, 4) if total else 0.0,
                "evictions": self.evictions,
                "rejected": self.rejected,
            }
            if self.arena is not None:
                out["arena_fallbacks"] = self.arena_fallbacks
                out["arena"] = self.arena.stats()
            return out

    def get(self, key: str) -> StateEntry | None:
        with self._lock:
            entry = self._entries.get(key)
            if entry is None:
                self.misses += 1
                return None
            entry.last_used = time.monotonic()
            entry.hits += 1
            self._entries.move_to_end(key)
            self.hits += 1
            return entry

    def put(self, key: str, snapshot: Any, state_len: int, media_hash: str = "") -> StateEntry | None:
        layout = SnapshotLayout.of(snapshot) if self.arena is not None else None
        nbytes = layout.tensor_bytes if layout is not None else tensor_bytes(snapshot)
        if self.capacity_bytes == 0 or nbytes > self.capacity_bytes:
            self.rejected += 1
            return None
        with self._lock:
            existing = self._entries.pop(key, None)
            if existing is not None:
                self._bytes -= existing.nbytes
            stored = snapshot
            if layout is not None:
                # the entries the reference's post-insert trim evicts, evicted before the copy
                self._trim(incoming=nbytes)
                packed = pack_snapshot(snapshot, self.arena, layout)
                if packed is None:
                    self.arena_fallbacks += 1
                else:
                    stored = packed
            self._entries[key] = StateEntry(
                key=key, snapshot=stored, state_len=int(state_len), nbytes=nbytes, media_hash=media_hash
            )
            self._bytes += nbytes
            self._trim()
            return self._entries.get(key)

    def acquire(self, key: str) -> StateEntry:
        with self._lock:
            entry = self._entries.get(key)
            if entry is None:
                raise StateCacheError(f"state {key} is not in the cache")
            entry.refcount += 1
            entry.last_used = time.monotonic()
            self._entries.move_to_end(key)
            return entry

    def release(self, key: str) -> None:
        with self._lock:
            entry = self._entries.get(key)
            if entry is not None and entry.refcount > 0:
                entry.refcount -= 1

    def drop(self, key: str) -> None:
        with self._lock:
            entry = self._entries.pop(key, None)
            if entry is not None:
                self._bytes -= entry.nbytes

    def clear(self) -> None:
        with self._lock:
            self._entries.clear()
            self._bytes = 0

    def _trim(self, incoming: int = 0) -> None:
        """Evict LRU-first while over budget; stop at an entry a running batch holds."""
        while self._bytes + incoming > self.capacity_bytes and self._entries:
            key, entry = next(iter(self._entries.items()))
            if entry.refcount > 0:
                break
            self._entries.pop(key, None)
            self._bytes -= entry.nbytes
            self.evictions += 1

    def get_or_compute(
        self,
        key: str,
        factory: Callable[[], tuple[Any, int]],
        *,
        media_hash: str = "",
    ) -> tuple[StateEntry, bool]:
        """``(entry, hit)``; on a miss the factory's snapshot is stored (cache.py:173-184).

        The new entry is returned without a reference; call ``acquire`` to keep it
        across an asynchronous batch.
        """
        entry = self.get(key)
        if entry is not None:
            return entry, True
        snapshot, state_len = factory()
        entry = self.put(key, snapshot, state_len, media_hash)
        if entry is None:
            entry = StateEntry(key=key, snapshot=snapshot, state_len=state_len, nbytes=tensor_bytes(snapshot))
        return entry, False


__all__ = ["PackedSnapshot", "SnapshotArena", "StateCache", "StateCacheError", "StateEntry", "tensor_bytes"]
