"""Overlapped host <-> device question passes against one resident state.

In the state-once serving loop the state K/V of a request stays on the GPU
while batches of question blocks arrive from the host and their attention
outputs go back to it (d3trt/model/trtllm_stack.py feeds one batch at a time
and waits for it). ``QuestionPipeline`` runs each batch as three stages on
three CUDA streams:

    host -> device copy of q, k_q, v_q   (copy-in stream)
    prefix_bidir_attention               (compute stream)
    device -> host copy of the output    (copy-out stream)

with ``depth`` sets of device buffers, so the copies of batch i+1 and i-1
overlap the attention of batch i. Host tensors must be pinned for the copies
to be asynchronous. Results are the same as calling ``prefix_bidir_attention``
on each batch in turn.

    pipe = QuestionPipeline(k_state, v_state, scale=D ** -0.5)
    for q, kq, vq, lengths, out in batches:      # pinned host tensors
        pipe.submit(q, kq, vq, lengths, out)
    pipe.synchronize()                           # every `out` is filled
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch

from .prefix_bidir import block_offsets, prefix_bidir_attention


class _Slot:
    """Device buffers of one batch in flight and the events that order their reuse."""

    def __init__(self) -> None:
        self.bufs: dict[str, torch.Tensor] = {}
        self.copied_in = torch.cuda.Event()
        self.computed = torch.cuda.Event()
        self.copied_out = torch.cuda.Event()
        self.used = False


class QuestionPipeline:
    """Question passes for a stream of host batches over one device-resident state."""

    def __init__(self, k_state: torch.Tensor, v_state: torch.Tensor, *, scale: float, depth: int = 2,
                 before_compute: Callable[[], None] | None = None):
        if not k_state.is_cuda or not v_state.is_cuda:
            raise RuntimeError("k_state/v_state must be device tensors (the state stays resident)")
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.k_state, self.v_state, self.scale = k_state, v_state, scale
        self.device = k_state.device
        self.copy_in = torch.cuda.Stream(self.device)
        self.compute = torch.cuda.Stream(self.device)
        self.copy_out = torch.cuda.Stream(self.device)
        self.slots = [_Slot() for _ in range(depth)]
        self.before_compute = before_compute  # optional work queued on the compute stream before each pass
        self.count = 0

    def _buf(self, slot: _Slot, name: str, like: torch.Tensor) -> torch.Tensor:
        b = slot.bufs.get(name)
        if b is None or b.shape != like.shape or b.dtype != like.dtype:
            with torch.cuda.stream(self.copy_in):
                b = torch.empty(like.shape, dtype=like.dtype, device=self.device)
            b.record_stream(self.compute)  # used on all three streams: not reused before they are done
            b.record_stream(self.copy_out)
            slot.bufs[name] = b
        return b

    def submit(self, q: torch.Tensor, k_q: torch.Tensor, v_q: torch.Tensor, lengths: Sequence[int] | torch.Tensor,
               out: torch.Tensor) -> torch.cuda.Event:
        """Queue one batch; returns the event recorded once its output is in ``out``.

        q [B, H, L, D], k_q / v_q [B, H_kv, L, D] and out [B, H, L, D] are host
        tensors (pinned, contiguous). The call returns once the work is queued.
        """
        slot = self.slots[self.count % len(self.slots)]
        self.count += 1
        lens = block_offsets(lengths, self.device)
        with torch.cuda.stream(self.copy_in):
            if slot.used:  # this slot's buffers are free once its previous output has left the GPU
                self.copy_in.wait_event(slot.copied_out)
            dq = self._buf(slot, "q", q)
            dkq = self._buf(slot, "kq", k_q)
            dvq = self._buf(slot, "vq", v_q)
            dout = self._buf(slot, "out", out)
            dq.copy_(q, non_blocking=True)
            dkq.copy_(k_q, non_blocking=True)
            dvq.copy_(v_q, non_blocking=True)
            slot.copied_in.record(self.copy_in)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(slot.copied_in)
            if self.before_compute is not None:
                self.before_compute()
            prefix_bidir_attention(dq, self.k_state, self.v_state, dkq, dvq, lens, scale=self.scale, out=dout)
            slot.computed.record(self.compute)
        with torch.cuda.stream(self.copy_out):
            self.copy_out.wait_event(slot.computed)
            out.copy_(dout, non_blocking=True)
            slot.copied_out.record(self.copy_out)
        slot.used = True
        return slot.copied_out

    def synchronize(self) -> None:
        """Wait until every submitted batch is back on the host."""
        self.copy_out.synchronize()
