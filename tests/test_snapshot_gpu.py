"""GPU parity of the packed snapshot format and the arena-backed state cache.

Packing is a byte copy, so every check is bit-exact: the packed block against
the packing oracle, the packed views against the tensors they came from, the
question pass on packed K/V against the same pass on the caller's views, a
round trip through pinned host memory, and the reference StateCache trace
replayed with an arena.
"""

from __future__ import annotations

import dataclasses
import gc
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import snapshot as osnap
from test_cache import _load_trace_module, _views

from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.kernels import prefix_bidir as pb
from d3_turbo_trt_b200.model import cache as dcache
from d3_turbo_trt_b200.model.snapshot import (
    AttentionEntry,
    DeltaEntry,
    PackedSnapshot,
    SnapshotArena,
    copy_segments,
    pack_snapshot,
)

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLDEN = Path(__file__).resolve().parent / "golden"


def _state_pass_like(layers_attn=2, layers_delta=3, S=1024, Hkv=4, D=128, conv=1280, Hv=6, seed=0):
    """Entries shaped and strided like D3Core's state pass leaves them (core.py:233-251, :301-358)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    snap = []
    for _ in range(layers_attn):
        k = torch.randn(1, S, Hkv, D, generator=g, device=DEV).to(torch.bfloat16).transpose(1, 2)
        v = torch.randn(1, S, Hkv * D, generator=g, device=DEV).to(torch.bfloat16).view(1, S, Hkv, D).transpose(1, 2)
        snap.append(AttentionEntry(keys=k, values=v))
    for _ in range(layers_delta):
        mixed = torch.randn(1, S, conv, generator=g, device=DEV).to(torch.bfloat16).transpose(1, 2)
        rec = torch.randn(1, Hv, 128, 128, generator=g, device=DEV)
        snap.append(DeltaEntry(tail=mixed[:, :, -3:], recurrent=rec))
    return snap


def _flat(snapshot):
    return [getattr(e, f.name) for e in snapshot for f in dataclasses.fields(e)]


def _same_view(t: torch.Tensor, device) -> torch.Tensor:
    """The same view (shape, strides, storage offset) over a copy of its whole storage on ``device``
    (``Tensor.to`` would make sliced and broadcast views contiguous)."""
    n = t.untyped_storage().nbytes() // t.element_size()
    if n == 0:
        return torch.empty(t.shape, dtype=t.dtype, device=device)
    whole = torch.as_strided(t, (n,), (1,), 0).to(device)
    return whole.as_strided(t.shape, t.stride(), t.storage_offset())


def _check_block(packed: PackedSnapshot, tensors):
    placed, total = osnap.pack([None if t is None else _same_view(t, "cpu") for t in tensors])
    raw = packed.block.bytes_view().cpu().numpy()
    assert packed.layout.nbytes == total
    for off, want in placed:
        assert np.array_equal(raw[off:off + len(want)], want)
    for t, v in zip(tensors, _flat(packed)):
        if t is None:
            assert v is None
            continue
        assert v.shape == t.shape and v.dtype == t.dtype and torch.equal(v, t)


def test_pack_matches_oracle_all_widths():
    """Strided, sliced, broadcast, empty, 0-d and misaligned tensors (16/8/4/2/1-byte paths)."""
    arena = SnapshotArena(1 << 20, DEV)
    for seed in range(3):
        tensors = [_same_view(t, DEV) for t in _views(seed)]
        tensors.append(None)
        snap = [AttentionEntry(keys=tensors[i], values=tensors[i + 1]) for i in range(0, len(tensors), 2)]
        packed = pack_snapshot(snap, arena)
        torch.cuda.synchronize()
        _check_block(packed, tensors)
    # odd byte offsets force the 8/4/2/1-byte accesses
    src = torch.arange(4096, device=DEV).to(torch.uint8)
    dst = torch.zeros(4096, dtype=torch.uint8, device=DEV)
    spec = [(8, 8, 1, 1, 1000, 0, 0, 0, 0), (1012, 1012, 1, 7, 12, 0, 20, 0, 12),
            (1202, 1202, 3, 5, 6, 50, 10, 30, 6), (1501, 1501, 1, 1, 999, 0, 0, 0, 0),
            (2600, 3600, 2, 3, 5, -300, 100, 20, 5)]
    copy_segments([_lib.CopySegment(src.data_ptr() + so, dst.data_ptr() + do, *rest) for so, do, *rest in spec], DEV)
    want = np.zeros(4096, np.uint8)
    osnap.apply_segments(np.arange(4096).astype(np.uint8), want, spec)
    assert np.array_equal(dst.cpu().numpy(), want)


def test_many_segments_span_launches():
    """More than one launch's worth of segments (128 per launch), mixed widths."""
    src = torch.arange(1 << 20, device=DEV).to(torch.uint8)
    dst = torch.zeros(1 << 20, dtype=torch.uint8, device=DEV)
    spec = [(i * 3000 + (i % 3), i * 3000 + (i % 3), 1, 2, 1000 + (i % 7) * 16, 0, 1200, 0, 1100) for i in range(300)]
    copy_segments([_lib.CopySegment(src.data_ptr() + so, dst.data_ptr() + do, *rest) for so, do, *rest in spec], DEV)
    want = np.zeros(1 << 20, np.uint8)
    osnap.apply_segments(np.arange(1 << 20).astype(np.uint8), want, spec)
    assert np.array_equal(dst.cpu().numpy(), want)


def test_pack_state_pass_snapshot_and_attention_reads_it():
    """A snapshot with views like the state pass's; the question pass gives identical bits on it."""
    snap = _state_pass_like()
    tensors = _flat(snap)
    arena = SnapshotArena(64 << 20, DEV)
    packed = pack_snapshot(snap, arena)
    assert isinstance(packed[0], AttentionEntry) and isinstance(packed[2], DeltaEntry)
    torch.cuda.synchronize()
    _check_block(packed, tensors)
    # the conv tail is 3 columns again, not its parent buffer
    assert packed.layout.tensor_bytes == dcache.tensor_bytes(snap)
    assert packed.layout.nbytes < sum(t.untyped_storage().nbytes() for t in tensors)
    g = torch.Generator(device=DEV).manual_seed(5)
    B, H, L, D = 4, 32, 64, 128
    q = torch.randn(B, H, L, D, generator=g, device=DEV).to(torch.bfloat16)
    kq = torch.randn(B, 4, L, D, generator=g, device=DEV).to(torch.bfloat16)
    vq = torch.randn(B, 4, L, D, generator=g, device=DEV).to(torch.bfloat16)
    lens = [64, 1, 37, 0]
    for e_src, e_pk in zip(snap[:2], packed[:2]):
        a = pb.prefix_bidir_attention(q, e_src.keys[0], e_src.values[0], kq, vq, lens, scale=D ** -0.5)
        b = pb.prefix_bidir_attention(q, e_pk.keys[0], e_pk.values[0], kq, vq, lens, scale=D ** -0.5)
        assert torch.equal(a, b)
    assert _lib.device_error() == 0


def test_block_lifetime_and_host_round_trip():
    snap = _state_pass_like(layers_attn=1, layers_delta=1, S=512)
    arena = SnapshotArena(8 << 20, DEV)
    packed = pack_snapshot(snap, arena)
    first = packed.block.offset
    host = packed.to_host()
    del packed
    gc.collect()
    torch.cuda.synchronize()
    assert arena.stats()["blocks"] == 0  # the block went back once its list was dropped
    restored = host.restore(arena)
    torch.cuda.synchronize()
    assert restored.block.offset == first
    for t, v in zip(_flat(snap), _flat(restored)):
        assert torch.equal(t, v)
    # no room: pack returns None and leaves the arena as it was
    small = SnapshotArena(4096, DEV)
    assert pack_snapshot(snap, small) is None and small.stats()["blocks"] == 0


@pytest.mark.parametrize("name", ["lru", "tight", "zero"])
def test_cache_with_arena_replays_reference_trace(name):
    """Same results, stats and LRU order as the reference, with every stored snapshot packed."""
    trace = json.loads((GOLDEN / "cache_trace.json").read_text())[name]
    gen = _load_trace_module()
    orig_snapshot_of = gen.snapshot_of
    gen.snapshot_of = lambda sizes: [torch.zeros(n, dtype=torch.float32, device=DEV) for n in sizes]
    try:
        arena = SnapshotArena(4 * trace["capacity"] + 4096, DEV)
        cache = dcache.StateCache(trace["capacity"], arena=arena)
        for i, step in enumerate(trace["steps"]):
            got = gen.apply(cache, step["call"], dcache.StateCacheError)
            assert got == step["result"], f"step {i} {step['call']}"
            assert gen.observe(cache) == step["after"], f"step {i} {step['call']}"
        packed = [e for e in cache.entries() if isinstance(e.snapshot, PackedSnapshot)]
        assert cache.count == 0 or packed
        assert arena.stats()["used_bytes"] >= sum(e.nbytes for e in packed)
    finally:
        gen.snapshot_of = orig_snapshot_of
