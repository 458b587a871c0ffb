"""Question-pass scheduling: batch bounds and CUDA-graph replay.

``state_once_batches(lengths, state)`` keeps the reference's batching
(reference/d3_runtime.py:1290-1314): question blocks sorted by length, a batch
closed when it would exceed 64 rows, 2^18 keys or 2^27 attention scores. Those
bounds exist because the reference's masked SDPA materialises every row's
keys and scores; ``prefix_bidir_attention`` materialises neither, so
``single_batch(lengths)`` (one launch for all blocks, still shortest first)
is the schedule this library's kernel wants.

``QuestionPassGraph`` captures one question pass for fixed shapes (rows,
width, heads) as a CUDA graph over static device buffers. A call then costs
one graph launch instead of the wrapper's checks, tensor-map encoding and
kernel launch; lengths (each <= width) and the data change between replays,
the shapes do not. Write the inputs into ``q``, ``k_q``, ``v_q`` (or pass
tensors to ``run``, which copies them in) and read ``out``.
"""

from __future__ import annotations

from typing import Sequence

import torch

from .prefix_bidir import prefix_bidir_attention

STATE_ONCE_ROWS = 64
STATE_ONCE_KEYS = 1 << 18
STATE_ONCE_SCORES = 1 << 27


def state_once_batches(lengths: Sequence[int], state: int) -> list[list[int]]:
    """Batches of question-block indices under the reference's bounds (d3_runtime.py:1297-1314):
    shortest blocks first; a block too large for the bounds still gets a batch of its own."""
    batches: list[list[int]] = []
    current: list[int] = []
    for i in sorted(range(len(lengths)), key=lambda j: lengths[j]):
        rows, widest = len(current) + 1, int(lengths[i])
        if current and (rows > STATE_ONCE_ROWS or rows * (state + widest) > STATE_ONCE_KEYS
                        or rows * widest * (state + widest) > STATE_ONCE_SCORES):
            batches.append(current)
            current = []
        current.append(i)
    if current:
        batches.append(current)
    return batches


def single_batch(lengths: Sequence[int]) -> list[list[int]]:
    """All blocks in one batch, shortest first: the kernel keeps no per-row key or score buffers."""
    return [sorted(range(len(lengths)), key=lambda j: lengths[j])] if len(lengths) else []


class QuestionPassGraph:
    """One question pass of fixed shapes captured as a CUDA graph; replays change data and lengths only."""

    def __init__(self, k_state: torch.Tensor, v_state: torch.Tensor, *, rows: int, width: int, heads: int,
                 scale: float):
        if not k_state.is_cuda:
            raise RuntimeError("QuestionPassGraph needs device tensors")
        kv_heads, _, dim = k_state.shape
        dev, dt = k_state.device, k_state.dtype
        self.k_state, self.v_state, self.scale = k_state, v_state, scale
        self.rows, self.width = rows, width
        self.q = torch.zeros(rows, heads, width, dim, dtype=dt, device=dev)
        self.k_q = torch.zeros(rows, kv_heads, width, dim, dtype=dt, device=dev)
        self.v_q = torch.zeros(rows, kv_heads, width, dim, dtype=dt, device=dev)
        self.out = torch.empty(rows, heads, width, dim, dtype=dt, device=dev)
        self.lengths = torch.full((rows,), width, dtype=torch.int32, device=dev)
        # pinned staging for host lengths: a small ring, each slot reused only after its copy finished
        self._stage = [torch.empty(rows, dtype=torch.int32, pin_memory=True) for _ in range(4)]
        self._stage_done = [None] * 4
        self._stage_next = 0
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._launch()  # first launch outside the capture: sets the kernel's shared-memory attribute
        side.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            self._launch()
        torch.cuda.current_stream(dev).wait_stream(side)

    def _launch(self) -> None:
        prefix_bidir_attention(self.q, self.k_state, self.v_state, self.k_q, self.v_q, self.lengths,
                               scale=self.scale, out=self.out)

    def set_lengths(self, lengths: Sequence[int] | torch.Tensor) -> None:
        """New real lengths (each in [0, width]); queued on the current stream before the next replay."""
        if isinstance(lengths, torch.Tensor) and lengths.is_cuda:
            self.lengths.copy_(lengths.to(torch.int32), non_blocking=True)
            return
        vals = [int(n) for n in (lengths.tolist() if isinstance(lengths, torch.Tensor) else lengths)]
        if len(vals) != self.rows or min(vals, default=0) < 0 or max(vals, default=0) > self.width:
            raise RuntimeError(f"lengths must be {self.rows} values in [0, {self.width}]")
        i = self._stage_next
        self._stage_next = (i + 1) % len(self._stage)
        if self._stage_done[i] is not None:
            self._stage_done[i].synchronize()
        self._stage[i].copy_(torch.tensor(vals, dtype=torch.int32))
        self.lengths.copy_(self._stage[i], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._stage_done[i] = ev

    def replay(self) -> torch.Tensor:
        """Run the captured pass on the current contents of q / k_q / v_q / lengths."""
        self.graph.replay()
        return self.out

    def run(self, q: torch.Tensor, k_q: torch.Tensor, v_q: torch.Tensor,
            lengths: Sequence[int] | torch.Tensor) -> torch.Tensor:
        """Copy the batch into the static buffers, then replay; returns the static output."""
        self.q.copy_(q, non_blocking=True)
        self.k_q.copy_(k_q, non_blocking=True)
        self.v_q.copy_(v_q, non_blocking=True)
        self.set_lengths(lengths)
        return self.replay()
