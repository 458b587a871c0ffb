"""Multi-GPU question-block sharding (one process per GPU, torch.distributed).

The state-once design has one exchange step: rank 0 runs the state pass and
broadcasts each full-attention layer's state K/V (and, end to end, the GDN
state) to every rank; the question blocks of the request are then split into
contiguous, length-sorted shards (the order of d3trt/backends/trtllm.py:149),
each rank runs its shard with no further communication, and the per-block
readout probabilities are gathered back. Independent requests are spread
data-parallel with no communication at all.

Collectives go through torch.distributed (NCCL over NVLink/NVSwitch on GPUs,
gloo on CPU for the tests). Every rank takes the same collective steps in the
same order. Received K/V lands in each rank's own HBM before any kernel reads
it; no kernel reads a peer's memory.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def nccl_options():
    """Options for the NCCL process group: collectives on high-priority streams.

    The attention kernels fill every SM with one CTA each, so a broadcast
    posted behind a state pass (StateKVExchange.post) waits for SMs; on a
    high-priority stream its CTAs take the next SM that frees up, ahead of the
    attention kernel's pending CTAs, and the layer moves while the next state
    pass runs."""
    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = True
    return opts


def shard_bounds(n_blocks: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous split of n_blocks into world_size shards of ceil/floor sizes.

    The first ``n_blocks % world_size`` ranks take one extra block, so shard
    sizes differ by at most one and every block is owned exactly once.
    """
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of {world_size}")
    base, extra = divmod(n_blocks, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def length_order(lengths: Sequence[int]) -> list[int]:
    """Block indices sorted by length, longest first (stable): shards get similar work."""
    return sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))


class StateKVExchange:
    """The state K/V of one request's full-attention layers, moved from ``src``
    to every rank one layer at a time (d3trt/model/core.py:150-154 produces
    them layer by layer in the state pass).

    Each layer's keys and values share one contiguous ``[2, S, Hkv, D]`` buffer
    (token-major, the layout the state pass writes and the question pass reads
    through strided views), so a layer crosses NVLink in a single broadcast.
    ``post(layer)`` enqueues that broadcast behind the work already queued on
    the current stream (on ``src``: the state pass that produced the layer)
    and returns at once: the next layer's state pass runs while NCCL moves this
    one. ``wait(layer)`` makes the current stream wait for the layer before a
    question pass reads it. Every rank posts every layer, in the same order.
    """

    def __init__(self, layers: int, tokens: int, kv_heads: int, head_dim: int, *, dtype: torch.dtype,
                 device: torch.device, src: int = 0, group=None):
        self.buffers = torch.empty((layers, 2, tokens, kv_heads, head_dim), dtype=dtype, device=device)
        self.src, self.group = src, group
        self._works: list = [None] * layers

    def kv(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(keys, values) of a layer as ``[Hkv, S, D]`` views (token-major strides)."""
        buf = self.buffers[layer]
        return buf[0].permute(1, 0, 2), buf[1].permute(1, 0, 2)

    def post(self, layer: int) -> None:
        if self._works[layer] is not None:
            raise RuntimeError(f"layer {layer} is already posted")
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            self._works[layer] = dist.broadcast(self.buffers[layer], src=self.src, group=self.group, async_op=True)
        else:
            self._works[layer] = True

    def wait(self, layer: int) -> None:
        work = self._works[layer]
        if work is None:
            raise RuntimeError(f"layer {layer} was never posted")
        if work is not True:
            work.wait()
        self._works[layer] = None


def broadcast_state_kv(entries: Sequence[tuple[torch.Tensor, torch.Tensor]], *, src: int = 0, group=None) -> None:
    """Broadcast every (keys, values) pair in place from ``src`` to all ranks.

    Non-source ranks pass preallocated tensors of the same shape/dtype; each
    tensor must be contiguous (NCCL moves flat buffers).
    """
    for k, v in entries:
        for t in (k, v):
            if not t.is_contiguous():
                raise ValueError("broadcast buffers must be contiguous")
            dist.broadcast(t, src=src, group=group)


def gather_rows(local: torch.Tensor, n_total: int, world_size: int, *, group=None) -> torch.Tensor:
    """All-gather per-rank row blocks (split by :func:`shard_bounds`) into [n_total, ...].

    Rows are padded to the largest shard for the collective and trimmed after.
    """
    biggest = -(-n_total // world_size)
    pad = torch.zeros((biggest, *local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world_size)]
    dist.all_gather(parts, pad, group=group)
    out = []
    for r in range(world_size):
        a, b = shard_bounds(n_total, world_size, r)
        out.append(parts[r][: b - a])
    return torch.cat(out, 0)


def sharded_question_pass(
    lengths: Sequence[int],
    run_blocks: Callable[[list[int]], torch.Tensor],
    *,
    rank: int,
    world_size: int,
    group=None,
) -> torch.Tensor:
    """Run this rank's shard of the (length-sorted) question blocks and gather.

    ``run_blocks(block_ids)`` returns one row per block in the given order
    (e.g. the readout probabilities). The result has one row per block in the
    original block order, identical on every rank.
    """
    order = length_order(lengths)
    a, b = shard_bounds(len(order), world_size, rank)
    mine = order[a:b]
    local = run_blocks(mine)
    if local.shape[0] != len(mine):
        raise RuntimeError(f"run_blocks returned {local.shape[0]} rows for {len(mine)} blocks")
    gathered = gather_rows(local, len(order), world_size, group=group) if world_size > 1 else local
    result = torch.empty_like(gathered)
    result[torch.tensor(order, device=gathered.device)] = gathered
    return result
