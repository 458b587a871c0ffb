"""Cross-request cache of state snapshots, budgeted in bytes (drop-in for
d3trt/model/cache.py:24-184: ``tensor_bytes``, ``StateEntry``, ``StateCache``).

The public surface and the observable rules are the reference's, because the
backend calls them (trtllm.py:131-147) and a recorded trace of the reference's
cache pins them (tests/golden/cache_trace.json): ``get`` / ``put`` / ``acquire``
/ ``release`` / ``drop`` / ``clear`` / ``get_or_compute`` / ``stats``; the least
recently used entry goes first; an entry held by ``acquire`` stops eviction
(the cache may then run over budget until it is released); a snapshot larger
than the budget is not stored.

How it is kept here: every use of an entry draws a ticket from a counter, and
a min-heap of (ticket, key) holds the recency order. Stale heap items (a key
used again since, or gone) are skipped when they reach the top and the heap is
rebuilt when they outnumber the live entries, so a use costs O(log n) and an
eviction looks at the oldest live ticket only.

With ``arena=SnapshotArena(...)`` each stored snapshot is packed into one block
of device memory (``pack_snapshot``: one copy launch), so the cache holds
exactly the bytes it counts, not the caller's tensors and the larger buffers
they may be views of. The entries that must go to make room are evicted before
the copy (the same ones the reference evicts after inserting), so the arena has
the space when the copy runs. If the arena still has no free range (its free
space is fragmented), the entry keeps the caller's tensors, as the reference's
does, and ``stats()["arena_fallbacks"]`` counts it.
"""

from __future__ import annotations

import heapq
import itertools
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable

from .snapshot import PackedSnapshot, SnapshotArena, SnapshotLayout, pack_snapshot


class StateCacheError(RuntimeError):
    """A cached state is missing, evicted while in use, or inconsistent."""


def tensor_bytes(obj: Any) -> int:
    """numel * element_size summed over every tensor reachable through lists, tuples and
    the attributes of objects (dataclasses with or without slots), as the reference counts."""
    total, pending = 0, [obj]
    while pending:
        item = pending.pop()
        if hasattr(item, "numel") and hasattr(item, "element_size"):
            total += int(item.numel()) * int(item.element_size())
        elif isinstance(item, (list, tuple)):
            pending.extend(item)
        elif hasattr(item, "__dict__"):
            pending.extend(vars(item).values())
        elif hasattr(item, "__slots__"):
            pending.extend(getattr(item, name) for name in item.__slots__ if hasattr(item, name))
    return total


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
    """Snapshots by state key under a byte budget; see the module docstring for the rules."""

    def __init__(self, capacity_bytes: int, *, arena: SnapshotArena | None = None):
        if capacity_bytes < 0:
            raise ValueError("capacity_bytes must be >= 0")
        self.capacity_bytes = int(capacity_bytes)
        self.arena = arena
        self._held: dict[str, StateEntry] = {}
        self._ticket: dict[str, int] = {}  # key -> ticket of its last use
        self._recency: list[tuple[int, str]] = []  # min-heap of (ticket, key), stale items included
        self._clock = itertools.count()
        self._used = 0
        self._lock = threading.RLock()
        self.hits = self.misses = self.evictions = self.rejected = self.arena_fallbacks = 0

    # ------------------------------------------------------------------ bookkeeping
    def _stamp(self, key: str) -> None:
        ticket = next(self._clock)
        self._ticket[key] = ticket
        heapq.heappush(self._recency, (ticket, key))
        if len(self._recency) > 4 * len(self._ticket) + 64:  # mostly stale: rebuild from the live tickets
            self._recency = [(t, k) for k, t in self._ticket.items()]
            heapq.heapify(self._recency)

    def _oldest(self) -> str | None:
        while self._recency:
            ticket, key = self._recency[0]
            if self._ticket.get(key) == ticket:
                return key
            heapq.heappop(self._recency)
        return None

    def _take(self, key: str) -> StateEntry | None:
        entry = self._held.pop(key, None)
        if entry is not None:
            del self._ticket[key]
            self._used -= entry.nbytes
        return entry

    def _make_room(self, incoming: int = 0) -> None:
        """Evict the least recently used entries until ``incoming`` more bytes fit; an entry
        a running batch holds (refcount > 0) stops the eviction where it stands."""
        while self._used + incoming > self.capacity_bytes:
            key = self._oldest()
            if key is None or self._held[key].refcount > 0:
                return
            self._take(key)
            self.evictions += 1

    # ------------------------------------------------------------------ queries
    @property
    def bytes(self) -> int:
        return self._used

    @property
    def count(self) -> int:
        return len(self._held)

    def __contains__(self, key: str) -> bool:
        with self._lock:
            return key in self._held

    def lru_keys(self) -> list[str]:
        """Keys from least to most recently used (the next eviction candidate first)."""
        with self._lock:
            return sorted(self._ticket, key=self._ticket.__getitem__)

    def entries(self) -> list[StateEntry]:
        with self._lock:
            return [self._held[k] for k in self.lru_keys()]

    def stats(self) -> dict[str, Any]:
        with self._lock:
            looked_up = self.hits + self.misses
            report = {"entries": len(self._held), "bytes": self._used, "capacity_bytes": self.capacity_bytes,
                      "hits": self.hits, "misses": self.misses,
                      "hit_rate": round(self.hits / looked_up, 4) if looked_up else 0.0,
                      "evictions": self.evictions, "rejected": self.rejected}
            if self.arena is not None:
                report["arena_fallbacks"] = self.arena_fallbacks
                report["arena"] = self.arena.stats()
            return report

    # ------------------------------------------------------------------ operations
    def get(self, key: str) -> StateEntry | None:
        with self._lock:
            entry = self._held.get(key)
            if entry is None:
                self.misses += 1
                return None
            self.hits += 1
            entry.hits += 1
            entry.last_used = time.monotonic()
            self._stamp(key)
            return entry

    def put(self, key: str, snapshot: Any, state_len: int, media_hash: str = "") -> StateEntry | None:
        layout = SnapshotLayout.of(snapshot) if self.arena is not None else None
        nbytes = tensor_bytes(snapshot) if layout is None else layout.tensor_bytes
        if self.capacity_bytes == 0 or nbytes > self.capacity_bytes:
            self.rejected += 1
            return None
        with self._lock:
            self._take(key)  # a re-put replaces the entry (no eviction is counted)
            stored = snapshot
            if layout is not None:
                self._make_room(nbytes)  # before the copy, so the arena has the space
                packed = pack_snapshot(snapshot, self.arena, layout)
                if packed is None:
                    self.arena_fallbacks += 1
                else:
                    stored = packed
            self._held[key] = StateEntry(key=key, snapshot=stored, state_len=int(state_len), nbytes=nbytes,
                                         media_hash=media_hash)
            self._used += nbytes
            self._stamp(key)
            self._make_room()
            return self._held.get(key)

    def acquire(self, key: str) -> StateEntry:
        with self._lock:
            entry = self._held.get(key)
            if entry is None:
                raise StateCacheError(f"state {key} is not in the cache")
            entry.refcount += 1
            entry.last_used = time.monotonic()
            self._stamp(key)
            return entry

    def release(self, key: str) -> None:
        with self._lock:
            entry = self._held.get(key)
            if entry is not None and entry.refcount:
                entry.refcount -= 1

    def drop(self, key: str) -> None:
        with self._lock:
            self._take(key)

    def clear(self) -> None:
        with self._lock:
            self._held.clear()
            self._ticket.clear()
            self._recency.clear()
            self._used = 0

    def get_or_compute(self, key: str, factory: Callable[[], tuple[Any, int]], *,
                       media_hash: str = "") -> tuple[StateEntry, bool]:
        """``(entry, hit)``. On a miss ``factory()`` -> ``(snapshot, state_len)`` is stored; a
        snapshot the cache rejects still comes back in an unstored entry. The entry is
        returned without a reference: ``acquire`` it to keep it across an asynchronous batch."""
        found = self.get(key)
        if found is not None:
            return found, True
        snapshot, state_len = factory()
        stored = self.put(key, snapshot, state_len, media_hash)
        if stored is not None:
            return stored, False
        return StateEntry(key=key, snapshot=snapshot, state_len=state_len, nbytes=tensor_bytes(snapshot)), False


__all__ = ["PackedSnapshot", "SnapshotArena", "StateCache", "StateCacheError", "StateEntry", "tensor_bytes"]
