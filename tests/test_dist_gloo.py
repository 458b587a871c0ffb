"""Question-block sharding on CPU ranks (gloo, world size 2): split coverage,
state-K/V broadcast, gather in original block order, and a rank that fails
mid-step (the survivor's collective ends with an error instead of hanging)."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from d3_turbo_trt_b200 import dist as d3dist


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_cover_every_block_once():
    for n in (0, 1, 7, 16, 255):
        for w in (1, 2, 3, 4, 8):
            spans = [d3dist.shard_bounds(n, w, r) for r in range(w)]
            owned = [i for a, b in spans for i in range(a, b)]
            assert owned == list(range(n))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        d3dist.shard_bounds(10, 2, 2)


def test_exchange_without_a_process_group_is_local():
    ex = d3dist.StateKVExchange(2, 16, 2, 8, dtype=torch.float32, device=torch.device("cpu"))
    ex.buffers.fill_(3.0)
    for layer in range(2):
        ex.post(layer)
    for layer in range(2):
        ex.wait(layer)
        k, v = ex.kv(layer)
        assert k.shape == (2, 16, 8) and torch.all(v == 3.0)
    with pytest.raises(RuntimeError):
        ex.wait(0)  # each post is waited once


def test_length_order_is_stable_longest_first():
    assert d3dist.length_order([3, 48, 48, 1, 20]) == [1, 2, 4, 0, 3]


def _worker(rank: int, world: int, port: int, scenario: str, q) -> None:
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from oracle import readout as oread

        g = torch.Generator().manual_seed(0)
        n_blocks, k, n_opt = 255, 64, 255
        hidden = torch.randn(n_blocks, k, generator=g)
        readout = torch.randn(n_opt, k, generator=g) * 0.1
        counts = [1 + (i * 37) % 255 for i in range(n_blocks)]
        lengths = [1 + (i * 11) % 48 for i in range(n_blocks)]

        # state K/V: rank 0 owns it, everyone else receives into its own buffer
        ks = torch.randn(4, 128, 32, generator=torch.Generator().manual_seed(5))
        vs = torch.randn(4, 128, 32, generator=torch.Generator().manual_seed(6))
        kb = ks.clone() if rank == 0 else torch.zeros_like(ks)
        vb = vs.clone() if rank == 0 else torch.zeros_like(vs)
        d3dist.broadcast_state_kv([(kb, vb)], src=0)
        assert torch.equal(kb, ks) and torch.equal(vb, vs)

        # per-layer exchange: every layer posted as it is produced, waited before use
        ex = d3dist.StateKVExchange(3, 128, 4, 32, dtype=torch.float32, device=torch.device("cpu"))
        for layer in range(3):
            if rank == 0:
                ex.buffers[layer].copy_(torch.full_like(ex.buffers[layer], float(layer + 1)))
                ex.buffers[layer, 0, 5, 2, 7] = -1.0
            else:
                ex.buffers[layer].zero_()
            ex.post(layer)
        for layer in range(3):
            ex.wait(layer)
            k, v = ex.kv(layer)
            assert k.shape == (4, 128, 32) and float(k[2, 5, 7]) == -1.0
            assert torch.all(v == layer + 1)

        def run_blocks(ids):
            if scenario == "fail" and rank == 1:
                raise RuntimeError("planted failure on rank 1")
            p = oread.probabilities(hidden[ids].numpy(), readout.numpy(), [counts[i] for i in ids], 1.0)
            return torch.from_numpy(p)

        full = d3dist.sharded_question_pass(lengths, run_blocks, rank=rank, world_size=world)
        ref = oread.probabilities(hidden.numpy(), readout.numpy(), counts, 1.0)
        assert np.array_equal(full.numpy(), ref)
        q.put((rank, "ok", ""))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, type(exc).__name__, "".join(traceback.format_exception_only(exc))))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(scenario: str, world: int = 2) -> dict[int, tuple[str, str]]:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, msg = q.get(timeout=120)
        results[rank] = (status, msg)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_sharded_pass_matches_single_rank():
    res = _run("ok")
    assert res == {0: ("ok", ""), 1: ("ok", "")}, res


def test_failing_rank_surfaces_as_error_not_hang():
    res = _run("fail")
    assert res[1][0] == "RuntimeError" and "planted failure" in res[1][1]
    assert res[0][0] != "ok"  # rank 0's gather ended with an error (peer gone / timeout)
