"""State snapshots packed into one HBM block: the format the state cache keeps.

A state pass leaves one entry per layer (d3trt/model/core.py:28-40):
``AttentionEntry(keys, values)``, each ``[1, Hkv, S, D]``, for the 16 full-attention
layers and ``DeltaEntry(tail, recurrent)`` (``[1, conv_dim, window]``,
``[1, Hv, Dk, Dv]``) for the 48 GDN layers. The reference caches that list as it is
(d3trt/model/cache.py:105-122), and its tensors are views: ``tail`` is the last
``window`` columns of the whole in_proj_qkv output (core.py:321), so each cached
GDN layer keeps a ``[S, conv_dim]`` buffer alive (80 MiB at S = 4096) while
``tensor_bytes`` (cache.py:24-34) counts 60 KiB for it.

``pack_snapshot`` copies every tensor of a snapshot into one block of a
``SnapshotArena`` with one ``d3b_copy_segments`` launch. Each tensor keeps its shape
and the order of its strides (a token-major K stays token-major, the layout the
attention kernel reads through TMA) and becomes dense, so a packed state holds
exactly its tensor bytes, 256-byte aligned per tensor. The result is a
``PackedSnapshot``: a list of entries of the same classes as the input (bare tensors
are entries too), which
``D3Core.questions`` and ``prefix_bidir_attention`` take unchanged.

Lifetime: a block goes back to the arena when the last reference to its
``PackedSnapshot`` list is dropped (keep the list, not single tensors, while a pass
uses them). The free waits for the work queued until then on the current stream
of the arena's device (a CUDA event), so a question pass still reading the block on
that stream is safe; readers on other streams must be ordered by the caller, as
for any tensor. Sources are read on the current stream at call time.
"""

from __future__ import annotations

import collections
import ctypes
import dataclasses
import functools
import itertools
import math
import threading
import weakref
from dataclasses import dataclass
from typing import Any, Sequence

import numpy as np
import torch

from .. import _lib

ALIGNMENT = 256
MAX_PIECES = 4096  # copy pieces one tensor may need before it counts as too fragmented


@dataclass(slots=True)
class AttentionEntry:
    keys: torch.Tensor  # [1, H_kv, S, D]
    values: torch.Tensor  # [1, H_kv, S, D]


@dataclass(slots=True)
class DeltaEntry:
    tail: torch.Tensor  # [1, conv_dim, window]
    recurrent: torch.Tensor  # [1, H_v, D_k, D_v]


Snapshot = list  # list[AttentionEntry | DeltaEntry]

# (src_offset, dst_offset, outer, rows, row_elems, src_outer, src_row, dst_outer, dst_row), in elements
Piece = tuple[int, int, int, int, int, int, int, int, int]


def plan_copy(shape: Sequence[int], strides: Sequence[int]) -> tuple[tuple[int, ...], list[Piece]]:
    """Packed (dense) strides for a tensor and the strided pieces that copy it there.

    Cached by (shape, strides): a 64-layer snapshot has a handful of distinct ones.

    The packed tensor orders its dimensions like the source (by stride, outermost
    first; equal strides keep index order), so a dense source is one contiguous
    piece. Source dimensions that are contiguous with respect to each other are
    merged; the innermost unit-stride run is a row, the next two dimensions are
    the piece's rows and outer count, and any further dimension is enumerated.
    """
    packed, pieces = _plan_copy(tuple(int(s) for s in shape), tuple(int(s) for s in strides))
    return packed, list(pieces)


@functools.lru_cache(maxsize=1024)
def _plan_copy(shape: tuple[int, ...], strides: tuple[int, ...]) -> tuple[tuple[int, ...], tuple[Piece, ...]]:
    ndim, numel = len(shape), math.prod(shape)
    if numel == 0:
        dense, p = [0] * ndim, 1
        for i in reversed(range(ndim)):
            dense[i] = p
            p *= max(shape[i], 1)
        return tuple(dense), ()
    order = sorted((i for i in range(ndim) if shape[i] > 1), key=lambda i: (-strides[i], i))
    packed, p = [numel] * ndim, 1
    for i in reversed(order):
        packed[i] = p
        p *= shape[i]
    merged: list[list[int]] = []  # [size, src stride, dst stride], outermost first
    for i in order:
        if merged and merged[-1][1] == strides[i] * shape[i]:
            merged[-1] = [merged[-1][0] * shape[i], strides[i], packed[i]]
        else:
            merged.append([shape[i], strides[i], packed[i]])
    row = merged.pop()[0] if merged and merged[-1][1] == 1 else 1
    if len(merged) > 2 and math.prod(d[0] for d in merged[:-2]) > MAX_PIECES:
        raise RuntimeError(f"tensor of shape {tuple(shape)} and strides {tuple(strides)} is too fragmented to pack")
    while len(merged) < 2:
        merged.insert(0, [1, 0, 0])
    (n_o, s_o, d_o), (n_r, s_r, d_r) = merged[-2], merged[-1]
    pieces: list[Piece] = []
    for idx in itertools.product(*(range(d[0]) for d in merged[:-2])):
        so = sum(k * d[1] for k, d in zip(idx, merged))
        do = sum(k * d[2] for k, d in zip(idx, merged))
        pieces.append((so, do, n_o, n_r, row, s_o, s_r, d_o, d_r))
    return tuple(packed), tuple(pieces)


def _fields(entry: Any) -> tuple[str, ...]:
    """Field names of an entry; a bare tensor entry has the one field ""."""
    if isinstance(entry, torch.Tensor):
        return ("",)
    if not dataclasses.is_dataclass(entry):
        raise TypeError(f"snapshot entries must be tensors or dataclasses of tensors, got {type(entry).__name__}")
    return tuple(f.name for f in dataclasses.fields(entry))


def _get(entry: Any, name: str) -> Any:
    return entry if name == "" else getattr(entry, name)


@dataclass(frozen=True, slots=True)
class Slot:
    entry: int
    field: str
    offset: int  # bytes from the start of the block
    nbytes: int
    shape: tuple[int, ...] | None  # None: the field held None
    strides: tuple[int, ...]
    dtype: torch.dtype | None
    pieces: tuple[Piece, ...]


class SnapshotLayout:
    """Where every tensor of a snapshot sits inside its packed block.

    ``segments`` holds every copy piece as one row of a ``d3b_copy_segment`` in
    bytes, with the source pointer and the block base still to be added
    (``piece_slot`` names each row's tensor), so packing builds its launch table
    with two vector adds.
    """

    def __init__(self, slots: list[Slot], types: list[type], nbytes: int):
        self.slots, self.types, self.nbytes = slots, types, nbytes
        rows, owner = [], []
        for i, s in enumerate(slots):
            if s.shape is None:
                continue
            es = s.dtype.itemsize
            for so, do, n_o, n_r, row, s_o, s_r, d_o, d_r in s.pieces:
                rows.append((so * es, s.offset + do * es, n_o, n_r, row * es, s_o * es, s_r * es, d_o * es, d_r * es))
                owner.append(i)
        self.segments = np.array(rows, dtype=np.int64).reshape(-1, 9)
        self.piece_slot = np.array(owner, dtype=np.int64)

    @classmethod
    def of(cls, snapshot: Sequence[Any]) -> "SnapshotLayout":
        """The layout of a snapshot; cached by the (entry class, shape, strides, dtype) signature."""
        sig = []
        for entry in snapshot:
            fields = _fields(entry)
            sig.append(torch.Tensor if isinstance(entry, torch.Tensor) else type(entry))
            for name in fields:
                t = _get(entry, name)
                sig.append((name, None) if t is None else (name, tuple(t.shape), t.stride(), t.dtype))
        key = tuple(sig)
        hit = _LAYOUTS.get(key)
        if hit is not None:
            _LAYOUTS.move_to_end(key)
            return hit
        slots, types, off, e = [], [], 0, -1
        for item in key:
            if isinstance(item, type):
                types.append(item)
                e += 1
                continue
            if item[1] is None:
                slots.append(Slot(e, item[0], off, 0, None, (), None, ()))
                continue
            name, shape, strides, dtype = item
            packed, pieces = _plan_copy(shape, tuple(strides))
            nb = math.prod(shape) * dtype.itemsize
            slots.append(Slot(e, name, off, nb, shape, packed, dtype, pieces))
            off += -(-nb // ALIGNMENT) * ALIGNMENT
        layout = cls(slots, types, max(off, ALIGNMENT))
        with _LAYOUTS_LOCK:
            _LAYOUTS[key] = layout
            while len(_LAYOUTS) > 64:
                _LAYOUTS.popitem(last=False)
        return layout

    @property
    def tensor_bytes(self) -> int:
        return sum(s.nbytes for s in self.slots)

    def table(self, snapshot: Sequence[Any], base: int) -> np.ndarray:
        """The ``d3b_copy_segment`` rows that copy ``snapshot`` into a block at device address ``base``."""
        src = np.zeros(len(self.slots), dtype=np.int64)
        for i, s in enumerate(self.slots):
            t = _get(snapshot[s.entry], s.field)
            if t is not None:
                src[i] = t.data_ptr()
        out = self.segments.copy()
        out[:, 0] += src[self.piece_slot]
        out[:, 1] += base
        return out


_LAYOUTS: collections.OrderedDict[tuple, SnapshotLayout] = collections.OrderedDict()
_LAYOUTS_LOCK = threading.Lock()


class _Block:
    """One live arena range; returns it to the arena when collected."""

    __slots__ = ("arena", "offset", "nbytes", "__weakref__")

    def __init__(self, arena: "SnapshotArena", offset: int, nbytes: int):
        self.arena, self.offset, self.nbytes = arena, offset, nbytes

    def bytes_view(self) -> torch.Tensor:
        return self.arena.buffer.narrow(0, self.offset, self.nbytes)

    def __del__(self):
        try:
            self.arena._release(self.offset)
        except Exception:  # interpreter shutdown: the arena goes with the process
            pass


class SnapshotArena:
    """One device buffer of ``capacity_bytes`` whose ranges the native allocator places.

    ``d3b_arena_*`` (best fit, coalescing, thread-safe) keeps the bookkeeping on the
    host; the buffer itself is a torch allocation made once.
    """

    def __init__(self, capacity_bytes: int, device: torch.device | str | int | None = None, *,
                 alignment: int = ALIGNMENT):
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("SnapshotArena needs a CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if capacity_bytes < 0:
            raise ValueError("capacity_bytes must be >= 0")
        lib = _lib.lib()
        handle = ctypes.c_void_p()
        _lib.check(lib.d3b_arena_create(int(capacity_bytes), int(alignment), ctypes.byref(handle)), "d3b_arena_create")
        self._handle = handle
        self._finalizer = weakref.finalize(self, lib.d3b_arena_destroy, handle)
        self.device, self.capacity_bytes, self.alignment = dev, int(capacity_bytes), int(alignment)
        self.buffer = torch.empty(self.capacity_bytes, dtype=torch.uint8, device=dev)
        self._lock = threading.RLock()
        self._pending: collections.deque[tuple[int, torch.cuda.Event]] = collections.deque()
        self._typed: dict[torch.dtype, torch.Tensor] = {}

    def typed(self, dtype: torch.dtype) -> torch.Tensor:
        """The whole buffer viewed as ``dtype`` (cached); element offsets are byte offsets / itemsize."""
        view = self._typed.get(dtype)
        if view is None:
            es = dtype.itemsize
            view = self.buffer[: self.capacity_bytes - self.capacity_bytes % es].view(dtype)
            self._typed[dtype] = view
        return view

    def allocate(self, nbytes: int) -> _Block | None:
        """A block of at least ``nbytes`` bytes, or None when no free range is large enough."""
        lib, off = _lib.lib(), ctypes.c_uint64()
        with self._lock:
            self._reap(wait=False)
            st = lib.d3b_arena_alloc(self._handle, int(nbytes), ctypes.byref(off))
            if st == _lib.ENOSPACE and self._pending:
                self._reap(wait=True)
                st = lib.d3b_arena_alloc(self._handle, int(nbytes), ctypes.byref(off))
        if st == _lib.ENOSPACE:
            return None
        _lib.check(st, "d3b_arena_alloc")
        return _Block(self, off.value, int(nbytes))

    def _release(self, offset: int) -> None:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._pending.append((offset, ev))  # deque.append is atomic: no lock from a finaliser

    def _reap(self, wait: bool) -> None:
        lib = _lib.lib()
        for _ in range(len(self._pending)):
            off, ev = self._pending.popleft()
            if wait:
                ev.synchronize()
            elif not ev.query():
                self._pending.append((off, ev))
                continue
            _lib.check(lib.d3b_arena_free(self._handle, off), "d3b_arena_free")

    def stats(self) -> dict[str, int]:
        with self._lock:
            self._reap(wait=False)
            out = (ctypes.c_uint64 * 4)()
            _lib.check(_lib.lib().d3b_arena_stats(self._handle, out), "d3b_arena_stats")
            return {"used_bytes": int(out[0]), "free_bytes": int(out[1]), "largest_free": int(out[2]),
                    "blocks": int(out[3]), "pending_frees": len(self._pending)}


class PackedSnapshot(list):
    """A snapshot whose tensors are views of one arena block; the block lives as long as this list."""

    __slots__ = ("block", "layout")

    @classmethod
    def _from_block(cls, block: _Block, layout: SnapshotLayout) -> "PackedSnapshot":
        fields: list[dict[str, Any]] = [{} for _ in layout.types]
        arena = block.arena
        for s in layout.slots:
            if s.shape is None:
                fields[s.entry][s.field] = None
            else:  # one as_strided over the arena viewed in the slot's dtype
                es = s.dtype.itemsize
                fields[s.entry][s.field] = torch.as_strided(arena.typed(s.dtype), s.shape, s.strides,
                                                            (block.offset + s.offset) // es)
        out = cls(kw[""] if typ is torch.Tensor else typ(**kw) for typ, kw in zip(layout.types, fields))
        out.block, out.layout = block, layout
        return out

    @property
    def nbytes(self) -> int:
        return self.layout.tensor_bytes

    def to_host(self) -> "HostSnapshot":
        """Copy the block to pinned host memory (one copy, queued on the current stream)."""
        host = torch.empty(self.layout.nbytes, dtype=torch.uint8, pin_memory=True)
        host.copy_(self.block.bytes_view()[: self.layout.nbytes], non_blocking=True)
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.block.arena.device))
        return HostSnapshot(host, self.layout, done)


class HostSnapshot:
    """A packed block in pinned host memory; ``restore`` brings it back with one copy."""

    def __init__(self, host: torch.Tensor, layout: SnapshotLayout, ready: torch.cuda.Event | None = None):
        self.host, self.layout, self._ready = host, layout, ready

    @property
    def nbytes(self) -> int:
        return self.layout.tensor_bytes

    def restore(self, arena: SnapshotArena) -> PackedSnapshot | None:
        block = arena.allocate(self.layout.nbytes)
        if block is None:
            return None
        stream = torch.cuda.current_stream(arena.device)
        if self._ready is not None:
            stream.wait_event(self._ready)
        block.bytes_view()[: self.layout.nbytes].copy_(self.host, non_blocking=True)
        return PackedSnapshot._from_block(block, self.layout)


def copy_segments(segments: Sequence[_lib.CopySegment] | np.ndarray, device: torch.device) -> None:
    """Run ``d3b_copy_segments`` on the current stream of ``device``.

    ``segments`` is a sequence of ``CopySegment`` or an int64 array [n, 9] with
    the same field order (pointers as integers).
    """
    if isinstance(segments, np.ndarray):
        arr = np.ascontiguousarray(segments, dtype=np.int64)
        n, ptr = arr.shape[0], arr.ctypes.data_as(ctypes.POINTER(_lib.CopySegment))
    else:
        n = len(segments)
        ptr = (_lib.CopySegment * n)(*segments)
    if n == 0:
        return
    with torch.cuda.device(device):
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        _lib.check(_lib.lib().d3b_copy_segments(ptr, n, stream), "d3b_copy_segments")


def pack_snapshot(snapshot: Sequence[Any], arena: SnapshotArena,
                  layout: SnapshotLayout | None = None) -> PackedSnapshot | None:
    """Copy a snapshot into one arena block (one launch); None when the arena has no room."""
    layout = layout or SnapshotLayout.of(snapshot)
    for s in layout.slots:
        t = _get(snapshot[s.entry], s.field)
        if t is not None and t.device != arena.device:
            raise RuntimeError(f"snapshot tensor on {t.device}, arena on {arena.device}")
    block = arena.allocate(layout.nbytes)
    if block is None:
        return None
    copy_segments(layout.table(snapshot, arena.buffer.data_ptr() + block.offset), arena.device)
    return PackedSnapshot._from_block(block, layout)
