"""Question-block sharding on 2 GPUs over NCCL (skipped with fewer GPUs).

Rank 0 owns the state K/V and broadcasts it with StateKVExchange; every rank
runs its contiguous, length-sorted shard of 255 ragged question blocks through
prefix_bidir_attention; the rows come back with gather_rows. The gathered
result must equal one GPU's pass over all 255 blocks bit for bit: each
(block, kv head, Q tile) unit is computed the same way whichever launch it
is in. NVLS is off (NCCL_NVLS_ENABLE=0) and every rank takes the same
collectives in the same order; the process group has a short timeout.
"""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B=255, H=32, Hkv=4, L=48, D=128, S=4096):
    g = torch.Generator().manual_seed(41)
    q = torch.randn(B, L, H, D, generator=g).to(torch.bfloat16)
    kq = torch.randn(B, L, Hkv, D, generator=g).to(torch.bfloat16)
    vq = torch.randn(B, L, Hkv, D, generator=g).to(torch.bfloat16)
    kv = torch.randn(2, S, Hkv, D, generator=g).to(torch.bfloat16)
    lengths = torch.randint(1, L + 1, (B,), generator=g).tolist()
    return q, kq, vq, kv, lengths


def _worker(rank: int, world: int, port: int, q_out) -> None:
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from d3_turbo_trt_b200 import _lib
        from d3_turbo_trt_b200 import dist as d3dist

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev,
                                pg_options=d3dist.nccl_options())
        from d3_turbo_trt_b200.kernels import prefix_bidir as pb

        q, kq, vq, kv, lengths = _inputs()
        B, L, H, D = q.shape
        Hkv, S = kq.shape[2], kv.shape[1]
        ex = d3dist.StateKVExchange(1, S, Hkv, D, dtype=torch.bfloat16, device=dev)
        if rank == 0:
            ex.buffers[0].copy_(kv)
        else:
            ex.buffers[0].zero_()
        ex.post(0)
        ex.wait(0)
        ks, vs = ex.kv(0)
        qd = q.to(dev).permute(0, 2, 1, 3)
        kqd = kq.to(dev).permute(0, 2, 1, 3)
        vqd = vq.to(dev).permute(0, 2, 1, 3)

        def run_blocks(ids):
            idx = torch.tensor(ids, device=dev)
            out = pb.prefix_bidir_attention(qd[idx], ks, vs, kqd[idx], vqd[idx], [lengths[i] for i in ids],
                                            scale=D ** -0.5)
            return out.reshape(len(ids), -1)

        full = d3dist.sharded_question_pass(lengths, run_blocks, rank=rank, world_size=world)
        torch.cuda.synchronize()
        if rank == 0:
            one = pb.prefix_bidir_attention(qd, kv[0].to(dev).permute(1, 0, 2), kv[1].to(dev).permute(1, 0, 2),
                                            kqd, vqd, lengths, scale=D ** -0.5).reshape(B, -1)
            assert torch.equal(full, one), float((full.float() - one.float()).abs().max())
        assert _lib.device_error() == 0
        q_out.put((rank, "ok", ""))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q_out.put((rank, type(exc).__name__, "".join(traceback.format_exception_only(exc))))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_question_pass_on_two_gpus_is_bit_exact():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, status, msg = q_out.get(timeout=300)
        results[rank] = (status, msg)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert results == {0: ("ok", ""), 1: ("ok", "")}, results
