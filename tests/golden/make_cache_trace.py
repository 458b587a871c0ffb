"""Record the reference StateCache's behaviour on seeded operation sequences.

    python tests/golden/make_cache_trace.py --reference <path to a d3-turbo-trt checkout>

(or set D3_REFERENCE_DIR). Drives d3trt.model.cache.StateCache (cache.py:50-184)
through random put / get / acquire / release / drop / contains / get_or_compute /
clear calls on snapshots of float32 tensors and writes, after every call, what it
returned, its stats() and the LRU order of its keys to cache_trace.json. The
tests replay the same calls on this library's StateCache and compare.
The fixture is committed; this script is only needed to regenerate it.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent

# (name, capacity bytes, calls, seed)
TRACES = [("lru", 6144, 400, 0), ("tight", 700, 80, 1), ("zero", 0, 20, 2)]


def snapshot_of(sizes):
    return [torch.zeros(n, dtype=torch.float32) for n in sizes]


def describe(entry):
    if entry is None:
        return None
    return {"key": entry.key, "state_len": entry.state_len, "nbytes": entry.nbytes,
            "refcount": entry.refcount, "hits": entry.hits, "media_hash": entry.media_hash}


def random_call(rng: random.Random):
    key = f"s{rng.randrange(12)}"
    r = rng.random()
    sizes = [64 * rng.randint(1, 6) for _ in range(rng.randint(1, 3))]
    if r < 0.33:
        return {"op": "put", "key": key, "sizes": sizes, "state_len": rng.randint(1, 9999),
                "media_hash": rng.choice(["", "m1"])}
    if r < 0.58:
        return {"op": "get", "key": key}
    if r < 0.68:
        return {"op": "acquire", "key": key}
    if r < 0.79:
        return {"op": "release", "key": key}
    if r < 0.84:
        return {"op": "drop", "key": key}
    if r < 0.89:
        return {"op": "contains", "key": key}
    if r < 0.985:
        return {"op": "get_or_compute", "key": key, "sizes": sizes, "state_len": rng.randint(1, 9999)}
    return {"op": "clear"}


def apply(cache, call, error_type):
    """Run one call; return a JSON-able description of its result."""
    op, key = call["op"], call.get("key")
    if op == "put":
        return describe(cache.put(key, snapshot_of(call["sizes"]), call["state_len"], call["media_hash"]))
    if op == "get":
        return describe(cache.get(key))
    if op == "acquire":
        try:
            return describe(cache.acquire(key))
        except error_type:
            return "raised"
    if op == "release":
        return cache.release(key)
    if op == "drop":
        return cache.drop(key)
    if op == "contains":
        return key in cache
    if op == "get_or_compute":
        calls = []

        def factory():
            calls.append(1)
            return snapshot_of(call["sizes"]), call["state_len"]

        entry, hit = cache.get_or_compute(key, factory)
        return {"entry": describe(entry), "hit": hit, "factory_calls": len(calls)}
    if op == "clear":
        return cache.clear()
    raise ValueError(op)


def observe(cache):
    stats = cache.stats()
    return {k: stats[k] for k in ("entries", "bytes", "capacity_bytes", "hits", "misses", "hit_rate",
                                  "evictions", "rejected")} | {"order": _lru_order(cache)}


def _lru_order(cache):
    """Keys least recently used first: the reference keeps them in an ordered dict; this
    library's cache reports them with lru_keys()."""
    return list(cache.lru_keys()) if hasattr(cache, "lru_keys") else list(cache._entries)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("D3_REFERENCE_DIR"))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference or set D3_REFERENCE_DIR")
    sys.path.insert(0, args.reference)
    from d3trt.errors import StateCacheError
    from d3trt.model.cache import StateCache

    out = {}
    for name, capacity, n, seed in TRACES:
        rng = random.Random(seed)
        cache = StateCache(capacity)
        steps = []
        for _ in range(n):
            call = random_call(rng)
            result = apply(cache, call, StateCacheError)
            steps.append({"call": call, "result": result, "after": observe(cache)})
        out[name] = {"capacity": capacity, "steps": steps}
    (HERE / "cache_trace.json").write_text(json.dumps(out, separators=(",", ":")))
    print({k: len(v["steps"]) for k, v in out.items()})


if __name__ == "__main__":
    main()
