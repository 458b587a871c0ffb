"""Host logic of the attention kernel's launch plan (no GPU needed).

d3b_prefix_bidir_ws runs one CTA per unit (block, head group, 128-row Q tile:
a kv head's whole GQA group, or a divisor of it when that gives fewer tiles)
and cuts the units of the last partial wave into pieces along their key tiles
(128 keys each, 64 for head_dim 256). The
piece that completes a unit merges the partial results through the workspace.
This file restates the plan (a greedy-dispatch model of the SMs) and checks
that the library's workspace size agrees with it. It then simulates the pieces
of each test shape in every arrival order: every slot and counter lies inside
the workspace, every unit's iterations are counted exactly once, exactly one
CTA writes each unit's rows, and the counters end at zero. The counts sit in a
region of the same size for every shape, so the partial slots of one shape
never overlap the counts of another. The library answers
these host-side queries without a GPU, with the B200's 148 SMs.
"""

from __future__ import annotations

import heapq
import random

import pytest

from d3_turbo_trt_b200 import _lib

BM = 128


def key_tile(D):
    """Keys per key tile: 64 for head_dim 256 (O takes 256 TMEM columns), else 128."""
    return 64 if D == 256 else 128
SMS = 148
CTA_COST = 12.0
MIN_SPLIT_TILES = 64
MAX_FULL_WAVES = 7


def tail_makespan(R, n, P, piece0, rest):
    sm = [0.0] * P
    mk, a, k = 0.0, 0, 0
    while a < n:
        ln = min(n - a, piece0 if k == 0 else rest)
        for _ in range(R):
            t = heapq.heappop(sm) + ln + CTA_COST
            mk = max(mk, t)
            heapq.heappush(sm, t)
        a += ln
        k += 1
    return mk


def plan(units, n, P=SMS):
    """(split_units, pieces, piece0, piece_rest); split_units == 0: no split."""
    R = units % P
    base = n + CTA_COST
    if R == 0 or n < MIN_SPLIT_TILES or units // P > MAX_FULL_WAVES or R > 256:
        return 0, 0, 0, 0
    best = None
    cands = [(t, n - t) for t in range((n + 1) // 2, n)]
    cands += [((n + k - 1) // k,) * 2 for k in range(3, min(8, n) + 1)]
    for p0, rest in cands:
        mk = tail_makespan(R, n, P, p0, rest)
        if best is None or mk < best[0]:
            best = (mk, p0, rest)
    mk, p0, rest = best
    pieces = 1 + (n - p0 + rest - 1) // rest
    if pieces > 1 and mk <= 0.97 * base:
        return R, pieces, p0, rest
    return 0, 0, 0, 0


def tile_shape(G, L):
    """(Gs, T, hsplit, token tiles): a Q tile holds Gs of a KV head's G query
    heads x T = BM // Gs tokens; Gs divides G and gives the fewest tiles per
    (block, KV head), ties to the largest Gs."""
    best = None
    for gs in range(G, 0, -1):
        if G % gs:
            continue
        T = BM // gs
        tiles = (L + T - 1) // T
        if best is None or (G // gs) * tiles < best[2] * best[3]:
            best = (gs, T, G // gs, tiles)
    return best


def shape(B, H, Hkv, S, L, D=128):
    _, T, hsplit, tiles = tile_shape(H // Hkv, L)
    BN = key_tile(D)
    return tiles, tiles * hsplit * Hkv * B, (S + BN - 1) // BN + (L + BN - 1) // BN, T


def ws_bytes(split, pieces, D):
    if not split:
        return 0
    # a fixed 1 KB count region for every shape, then one partial slot per piece
    return 1024 + split * pieces * (BM * D + 2 * BM) * 4


CASES = [
    ("cfg1", 8, 8, 2, 512, 32, 64),
    ("cfg3a", 16, 32, 4, 4096, 64, 128),
    ("cfg3b", 255, 32, 4, 16384, 48, 128),
    ("cfg5", 255, 32, 4, 16384, 64, 128),
    ("cfg5_rank_of_8", 32, 32, 4, 16384, 64, 128),
    ("state4k", 1, 32, 4, 0, 4096, 128),
    ("ragged_L300", 40, 16, 2, 300, 300, 64),
    ("g3", 200, 6, 2, 130, 20, 64),
    ("split_test", 300, 32, 4, 520, 64, 128),
    ("ragged_g6", 21, 24, 4, 700, 48, 128),
    ("cfg1_ragged_test", 8, 8, 2, 512, 32, 64),
    ("gpu_split_d64", 40, 8, 2, 8200, 300, 64),
    ("gpu_split_d128", 24, 32, 4, 8192, 64, 128),
    ("gpu_split_g6", 21, 24, 4, 8192, 48, 128),
    ("gpu_split_g6_L64", 16, 24, 4, 8192, 64, 128),
    ("model_g6_L64", 16, 24, 4, 4096, 64, 128),
    ("g12_L64", 37, 24, 2, 2048, 64, 128),
    ("g10_L50", 5, 20, 2, 700, 50, 128),
    ("model_d256", 16, 24, 4, 4096, 64, 256),
    ("d256_g1", 40, 4, 4, 3000, 40, 256),
    ("d256_ragged_L300", 3, 24, 4, 2000, 300, 256),
]


def test_tile_shape_fills_rows_when_the_group_does_not_divide_the_tile():
    # G = 8 (and every power of two): the whole group, 16 tokens per tile
    assert tile_shape(8, 64) == (8, 16, 1, 4)
    assert tile_shape(8, 4096) == (8, 16, 1, 256)
    # G = 6 at 64 tokens: 3 tiles of 2 heads x 64 tokens, not 4 of 6 heads x 21 tokens
    assert tile_shape(6, 64) == (2, 64, 3, 1)
    # G = 6 at 48 tokens: a tie (3 tiles either way) keeps the whole group
    assert tile_shape(6, 48) == (6, 21, 1, 3)
    # G = 12 at 64 tokens: 3 groups of 4 heads x 32 tokens (6 tiles; 7 for the whole group)
    assert tile_shape(12, 64) == (4, 32, 3, 2)
    # G = 10 at 50 tokens: 2 groups of 5 heads x 25 tokens (4 tiles, 125 of 128 rows; 5 for the group)
    assert tile_shape(10, 50) == (5, 25, 2, 2)
    assert tile_shape(3, 20) == (3, 42, 1, 1)


@pytest.mark.parametrize("name,B,H,Hkv,S,L,D", CASES)
def test_workspace_size_matches_plan(name, B, H, Hkv, S, L, D):
    _, units, n, _ = shape(B, H, Hkv, S, L, D)
    split, pieces, _, _ = plan(units, n)
    assert int(_lib.lib().d3b_prefix_bidir_workspace_size(B, H, Hkv, S, L, D)) == ws_bytes(split, pieces, D)


def test_long_units_are_cut_short_ones_are_not():
    # config 3a: 33-tile units; pieces would cost more than the 40 idle SMs of the last wave
    assert plan(*shape(16, 32, 4, 4096, 64)[1:3]) == (0, 0, 0, 0)
    # configs 3b and 5 on one GPU: 20+ full waves, the tail is a few per cent at most
    assert plan(*shape(255, 32, 4, 16384, 48)[1:3]) == (0, 0, 0, 0)
    # the GPU tests' split shapes are cut
    for B, H, Hkv, S, L in ((40, 8, 2, 8200, 300), (24, 32, 4, 8192, 64), (21, 24, 4, 8192, 48)):
        assert plan(*shape(B, H, Hkv, S, L)[1:3])[0] > 0
    # a rank's 32-block shard of config 5 (129-tile units, 3.46 waves): the last wave is cut
    _, units, n, _ = shape(32, 32, 4, 16384, 64)
    split, pieces, p0, rest = plan(units, n)
    assert (units, n) == (512, 129) and split == 512 - 3 * 148 and pieces >= 2
    assert tail_makespan(split, n, SMS, p0, rest) < 0.75 * (n + CTA_COST)


@pytest.mark.parametrize("name,B,H,Hkv,S,L,D", CASES)
def test_pieces_cover_every_unit_once(name, B, H, Hkv, S, L, D):
    tiles, units, n_full, T = shape(B, H, Hkv, S, L, D)
    BN = key_tile(D)
    split, pieces, p0, rest = plan(units, n_full)
    whole = units - split
    groups = units // (tiles * B)  # head groups: KV heads x hsplit
    n_s = (S + BN - 1) // BN
    slots = split * pieces
    rng = random.Random(hash(name) & 0xFFFF)
    for trial in range(4):
        lens = [L if trial == 0 else rng.randint(0, L) for _ in range(B)]
        ctas = list(range(whole + slots))
        rng.shuffle(ctas)  # any arrival order
        count = [0] * max(split, 1)
        counted = [0] * units
        writes = [0] * units
        for bid in ctas:
            if bid < whole:
                u, a, e, slot = bid, 0, n_full, -1
            else:
                q = bid - whole
                k, r = divmod(q, split)
                u, slot = whole + r, q
                a = 0 if k == 0 else p0 + (k - 1) * rest
                e = p0 if k == 0 else min(n_full, a + rest)
                assert 0 <= a < e <= n_full
                assert 0 <= slot < slots and 0 <= r < split
            tile, b = u % tiles, u // (tiles * groups)
            lb = min(max(lens[b], 0), L)
            counted[u] += e - a
            if tile * T >= lb:  # no real token: rows zeroed by the unit's first piece only
                writes[u] += a == 0
                continue
            cnt = max(0, min(e, n_s + (lb + BN - 1) // BN) - a)
            if slot < 0:
                assert cnt >= 1
                writes[u] += 1
                continue
            count[u - whole] += e - a
            if count[u - whole] == n_full:
                count[u - whole] = 0
                writes[u] += 1
        assert counted == [n_full] * units
        assert writes == [1] * units
        assert not any(count)


def test_workspace_size_matches_plan_on_random_shapes():
    """The library's tile shape and split plan against this file's restatement
    on 300 seeded shapes: GQA groups 1..16 (dividing 128 or not), every head
    dim, short and long blocks, with and without a state."""
    rng = random.Random(20261202)
    for _ in range(300):
        Hkv = rng.choice([1, 2, 4, 8])
        G = rng.randint(1, 16)
        B = rng.randint(1, 300)
        L = rng.choice([rng.randint(1, 64), rng.randint(65, 600)])
        S = rng.choice([0, rng.randint(1, 20000)])
        D = rng.choice([32, 64, 128, 256])
        _, units, n, _ = shape(B, G * Hkv, Hkv, S, L, D)
        if units > 0x7FFFFFFF:
            continue
        split, pieces, _, _ = plan(units, n)
        got = int(_lib.lib().d3b_prefix_bidir_workspace_size(B, G * Hkv, Hkv, S, L, D))
        assert got == ws_bytes(split, pieces, D), (B, G * Hkv, Hkv, S, L, D)
