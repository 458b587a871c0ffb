"""State cache and packed-snapshot host logic (CPU).

* The reference StateCache's recorded behaviour (tests/golden/cache_trace.json,
  made by make_cache_trace.py from d3trt/model/cache.py) replayed call by call
  on this library's StateCache: same results, stats and LRU order.
* The known-answer cases of the reference's own cache tests (LRU order,
  refcount pinning, get_or_compute hits, a budget too small).
* The copy-piece planner against the packing oracle, on strided, transposed,
  sliced, broadcast and empty tensors, through a CPU interpreter of the
  d3b_copy_segments semantics.
* The native arena allocator through the C ABI (no device memory involved).
"""

from __future__ import annotations

import ctypes
import json
import random
from pathlib import Path

import numpy as np
import pytest
import torch

from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.model import cache as dcache
from d3_turbo_trt_b200.model.snapshot import ALIGNMENT, AttentionEntry, DeltaEntry, SnapshotLayout, plan_copy
from oracle import snapshot as osnap

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load_trace_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_cache_trace", GOLDEN / "make_cache_trace.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("name", ["lru", "tight", "zero"])
def test_replays_reference_trace(name):
    trace = json.loads((GOLDEN / "cache_trace.json").read_text())[name]
    gen = _load_trace_module()
    cache = dcache.StateCache(trace["capacity"])
    for i, step in enumerate(trace["steps"]):
        got = gen.apply(cache, step["call"], dcache.StateCacheError)
        assert got == step["result"], f"step {i} {step['call']}: {got} != {step['result']}"
        assert gen.observe(cache) == step["after"], f"step {i} {step['call']}"


class _FakeArena:
    """Host stand-in for SnapshotArena: tracks bytes only (the copy itself needs a GPU)."""

    def __init__(self, capacity):
        self.capacity, self.used, self.live = capacity, 0, {}

    def stats(self):
        return {"used_bytes": self.used}


@pytest.mark.parametrize("name", ["lru", "tight"])
def test_arena_mode_evicts_like_the_reference(name, monkeypatch):
    """With an arena the eviction set is chosen before the copy; it must equal the reference's
    post-insert trim, and a full arena falls back to keeping the caller's tensors."""
    trace = json.loads((GOLDEN / "cache_trace.json").read_text())[name]
    gen = _load_trace_module()
    arena = _FakeArena(3 * max(trace["capacity"], 1))

    class Packed(list):
        def __del__(self):
            arena.used -= self.nbytes

    def fake_pack(snapshot, arena_, layout):
        assert arena_ is arena
        if arena.used + layout.nbytes > arena.capacity:
            return None
        out = Packed(snapshot)
        out.nbytes = layout.nbytes
        arena.used += layout.nbytes
        return out

    monkeypatch.setattr(dcache, "pack_snapshot", fake_pack)
    cache = dcache.StateCache(trace["capacity"], arena=arena)
    for i, step in enumerate(trace["steps"]):
        got = gen.apply(cache, step["call"], dcache.StateCacheError)
        assert got == step["result"], f"step {i} {step['call']}"
        assert gen.observe(cache) == step["after"], f"step {i} {step['call']}"
    stats = cache.stats()
    assert stats["arena"]["used_bytes"] == arena.used and "arena_fallbacks" in stats


def test_tensor_bytes_nested():
    payload = [torch.zeros(2, 3, dtype=torch.float32), (torch.zeros(4, dtype=torch.float16),)]
    assert dcache.tensor_bytes(payload) == 2 * 3 * 4 + 4 * 2
    entry = DeltaEntry(tail=torch.zeros(1, 6, 3, dtype=torch.bfloat16), recurrent=torch.zeros(1, 2, 4, 4))
    assert dcache.tensor_bytes([entry]) == 36 + 128


def test_lru_eviction_order():
    cache = dcache.StateCache(64)
    assert cache.put("a", [torch.zeros(8)], 1) is not None
    assert cache.put("b", [torch.zeros(8)], 1) is not None
    assert cache.bytes == 64
    assert cache.get("a") is not None
    assert cache.put("c", [torch.zeros(8)], 1) is not None  # b is the LRU entry now
    assert "a" in cache and "b" not in cache and "c" in cache
    assert cache.evictions == 1


def test_pinned_entry_survives():
    cache = dcache.StateCache(64)
    cache.put("a", [torch.zeros(8)], 1)
    cache.acquire("a")
    cache.put("b", [torch.zeros(8)], 1)
    cache.put("c", [torch.zeros(8)], 1)
    assert "a" in cache
    cache.release("a")
    cache.put("d", [torch.zeros(8)], 1)
    assert "a" not in cache or cache.bytes <= cache.capacity_bytes


def test_get_or_compute_and_small_budget():
    cache = dcache.StateCache(1024)
    calls = []

    def factory():
        calls.append(1)
        return [torch.ones(2, 2)], 3

    entry, hit = cache.get_or_compute("k", factory)
    assert not hit and entry.state_len == 3 and len(calls) == 1
    entry2, hit2 = cache.get_or_compute("k", factory)
    assert hit2 and entry2 is entry and len(calls) == 1
    tiny = dcache.StateCache(1)
    entry, hit = tiny.get_or_compute("k", lambda: ([torch.ones(2, 2)], 2))
    assert not hit and entry.nbytes == 16 and tiny.count == 0
    with pytest.raises(dcache.StateCacheError):
        tiny.acquire("missing")
    with pytest.raises(ValueError):
        dcache.StateCache(-1)


def _views(seed: int):
    """Tensors shaped like snapshot fields, as the state pass leaves them (views included)."""
    g = torch.Generator().manual_seed(seed)
    S, Hkv, D, conv, Hv = 37, 2, 16, 40, 3
    out = []
    k = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16).transpose(1, 2)  # token-major view
    out.append(k)
    qkv = torch.randn(1, S, 3 * Hkv * D, generator=g).to(torch.bfloat16)
    out.append(qkv[..., Hkv * D: 2 * Hkv * D].view(1, S, Hkv, D).transpose(1, 2))  # slice of a fused output
    mixed = torch.randn(1, S, conv, generator=g).to(torch.bfloat16).transpose(1, 2)
    out.append(mixed[:, :, -3:])  # the GDN conv tail view
    out.append(torch.randn(1, Hv, 8, 8, generator=g))  # recurrent state, fp32 contiguous
    out.append(torch.randn(5, 7, generator=g).t())  # plain transpose
    out.append(torch.randn(4, 1, 6, generator=g).expand(4, 3, 6))  # broadcast (stride 0)
    out.append(torch.randn(6, 10, generator=g)[::2, 1:8:3])  # step slices: element rows
    out.append(torch.randn(3, 4, 5, 6, generator=g).permute(2, 0, 3, 1)[1:4, :, 2:5])  # 4-d, many pieces
    out.append(torch.zeros(0, 5))  # empty
    out.append(torch.tensor(3.5))  # 0-d
    out.append(torch.randn(2, 3, generator=g).to(torch.float16)[:, 1:])  # misaligned start
    return out


def test_plan_matches_oracle():
    for seed in range(3):
        tensors = _views(seed)
        placed, total = osnap.pack(tensors)
        block = np.zeros(total, np.uint8)
        for t, (off, want) in zip(tensors, placed):
            packed_strides, pieces = plan_copy(t.shape, t.stride())
            es = t.element_size()
            base = t.storage_offset() * es
            storage = np.frombuffer(bytes(t.untyped_storage()), np.uint8)
            segs = [(base + so * es, off + do * es, n_o, n_r, row * es, s_o * es, s_r * es, d_o * es, d_r * es)
                    for so, do, n_o, n_r, row, s_o, s_r, d_o, d_r in pieces]
            osnap.apply_segments(storage, block, segs)
            assert np.array_equal(block[off:off + len(want)], want), (t.shape, t.stride())
            # the packed strides describe the same logical tensor over the packed bytes
            if t.numel():
                raw = torch.from_numpy(block[off:off + len(want)].copy()).view(t.dtype)
                view = torch.as_strided(raw, t.shape, packed_strides)
                assert torch.equal(view, t)


def test_layout_offsets_and_bytes():
    tensors = _views(7)
    snap = [AttentionEntry(tensors[0], tensors[1]), DeltaEntry(tensors[2], tensors[3])]
    layout = SnapshotLayout.of(snap)
    placed, total = osnap.pack(tensors[:4])
    assert [s.offset for s in layout.slots] == [p[0] for p in placed]
    assert layout.nbytes == total and all(s.offset % ALIGNMENT == 0 for s in layout.slots)
    # packed bytes are the tensor bytes: the tail no longer stands for its whole parent buffer
    assert layout.tensor_bytes == dcache.tensor_bytes(snap)
    assert tensors[2].untyped_storage().nbytes() > 10 * tensors[2].numel() * tensors[2].element_size()


def test_layout_of_bare_tensors_and_cache_keys():
    """Entries may be bare tensors (the reference cache takes any tensor list); layouts are cached."""
    snap = [torch.zeros(64), torch.zeros(3, 5).t(), DeltaEntry(torch.zeros(1, 4, 3), None)]
    a, b = SnapshotLayout.of(snap), SnapshotLayout.of([torch.ones(64), torch.ones(3, 5).t(), snap[2]])
    assert a is b and a.types == [torch.Tensor, torch.Tensor, DeltaEntry]
    assert [s.offset for s in a.slots] == [0, 256, 512, 768] and a.tensor_bytes == 256 + 60 + 48
    assert SnapshotLayout.of([torch.zeros(64, dtype=torch.float64)]) is not a


def test_packed_views_read_the_packed_bytes():
    """PackedSnapshot views over a block filled by the packing oracle equal the source tensors."""
    from d3_turbo_trt_b200.model import snapshot as sn

    tensors = _views(3)
    tensors.append(None)
    snap = [AttentionEntry(tensors[i], tensors[i + 1]) for i in range(0, len(tensors), 2)]
    layout = SnapshotLayout.of(snap)

    class Arena:  # host stand-in: the views only need the buffer and its typed views
        typed = sn.SnapshotArena.typed

        def __init__(self, nbytes):
            self.capacity_bytes, self._typed = nbytes, {}
            self.buffer = torch.zeros(nbytes, dtype=torch.uint8)

    class Block:
        def __init__(self, arena, offset):
            self.arena, self.offset = arena, offset

    arena = Arena(layout.nbytes + 1024)
    placed, _ = osnap.pack(tensors)
    buf = arena.buffer.numpy()
    for off, want in placed:
        buf[512 + off: 512 + off + len(want)] = want
    packed = sn.PackedSnapshot._from_block(Block(arena, 512), layout)
    for e_src, e_pk in zip(snap, packed):
        for name in ("keys", "values"):
            a, b = getattr(e_src, name), getattr(e_pk, name)
            assert (a is None and b is None) or (a.shape == b.shape and torch.equal(a, b))


def test_dense_tensor_is_one_piece():
    t = torch.zeros(1, 64, 4, 128, dtype=torch.bfloat16).transpose(1, 2)  # token-major K
    packed, pieces = plan_copy(t.shape, t.stride())
    assert packed == tuple(t.stride()) and len(pieces) == 1
    assert pieces[0][2:5] == (1, 1, t.numel())


def test_too_fragmented_raises():
    # five dimensions none of which merge: 100 x 100 pieces of 2 x 10 rows
    with pytest.raises(RuntimeError):
        plan_copy([3, 100, 100, 2, 10], [1, 10**7, 10**5, 1000, 10])
    assert len(plan_copy([3, 100, 2, 10], [1, 10**5, 1000, 10])[1]) == 100


class _Arena:
    def __init__(self, capacity, align=256):
        self.lib = _lib.lib()
        self.h = ctypes.c_void_p()
        _lib.check(self.lib.d3b_arena_create(capacity, align, ctypes.byref(self.h)), "create")

    def alloc(self, n):
        off = ctypes.c_uint64()
        st = self.lib.d3b_arena_alloc(self.h, n, ctypes.byref(off))
        return off.value if st == 0 else st

    def free(self, off):
        return self.lib.d3b_arena_free(self.h, off)

    def stats(self):
        out = (ctypes.c_uint64 * 4)()
        _lib.check(self.lib.d3b_arena_stats(self.h, out), "stats")
        return list(out)

    def close(self):
        self.lib.d3b_arena_destroy(self.h)


def test_arena_best_fit_coalesce_and_errors():
    a = _Arena(4096)
    try:
        x, y, z = a.alloc(1000), a.alloc(256), a.alloc(1)
        assert (x, y, z) == (0, 1024, 1280)
        assert a.stats() == [1024 + 256 + 256, 4096 - 1536, 4096 - 1536, 3]
        assert a.free(y) == 0 and a.free(y) == _lib.EINVAL  # double free is refused
        assert a.alloc(200) == 1024  # best fit: the 256-byte hole, not the tail
        assert a.alloc(5000) == _lib.ENOSPACE
        assert a.alloc(0) == _lib.EINVAL
        assert a.free(1024) == 0 and a.free(0) == 0 and a.free(1280) == 0
        assert a.stats() == [0, 4096, 4096, 0]  # everything coalesced back into one range
    finally:
        a.close()
    h = ctypes.c_void_p()
    assert _lib.lib().d3b_arena_create(4096, 100, ctypes.byref(h)) == _lib.EINVAL  # not a power of two


def test_arena_random_against_model():
    """Random alloc/free against a byte-map model: blocks never overlap and the stats add up."""
    cap, align = 1 << 16, 256
    a = _Arena(cap, align)
    rng = random.Random(0)
    live: dict[int, int] = {}
    try:
        for _ in range(3000):
            if live and rng.random() < 0.45:
                off = rng.choice(list(live))
                assert a.free(off) == 0
                del live[off]
            else:
                n = rng.randint(1, 6000)
                off = a.alloc(n)
                need = -(-n // align) * align
                if off == _lib.ENOSPACE:
                    assert a.stats()[2] < need
                    continue
                assert off % align == 0 and off + need <= cap
                assert all(off + need <= o or o + s <= off for o, s in live.items())
                live[off] = need
            used, free, largest, blocks = a.stats()
            assert used == sum(live.values()) and used + free == cap and blocks == len(live)
    finally:
        a.close()
