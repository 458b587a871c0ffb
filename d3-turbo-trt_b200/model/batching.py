"""Question ids of a request, built for the device with one copy per batch.

The reference's TRT-LLM backend (d3trt/backends/trtllm.py:149-162) orders a
request's question pieces by length, cuts the order into batches of
``d3.batch_size`` rows, and builds each batch's ids on the device as
``torch.full((rows, width), pad_id)`` followed by one host-to-device copy per
row (``ids[r, :len(piece)] = torch.as_tensor(piece, device=...)``): a fill
launch plus ``rows`` small synchronous copies per batch.

``QuestionBatcher`` produces the same tensors from the same pieces: each
batch's padded ``[rows, width]`` int64 ids and its int32 lengths are written
into one reusable pinned host buffer and moved with a single non-blocking
copy, so the host thread does not wait on the GPU and the copy overlaps the
previous batch's work on the stream. The staging buffer is reused only after
the copy that read it has completed (a CUDA event per buffer, two buffers in
rotation), so a batch's host memory is never overwritten while its copy is in
flight.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, Sequence

import numpy as np
import torch


def length_order(pieces: Sequence[Sequence[int]]) -> list[int]:
    """Indices of the pieces, shortest first; ties keep their order (trtllm.py:149, a stable sort)."""
    return sorted(range(len(pieces)), key=lambda i: len(pieces[i]))


def batch_orders(pieces: Sequence[Sequence[int]], batch_size: int) -> list[list[int]]:
    """The reference's batches: the length order cut into runs of ``max(1, batch_size)`` rows
    (trtllm.py:150-153)."""
    order = length_order(pieces)
    size = max(1, int(batch_size))
    return [order[s:s + size] for s in range(0, len(order), size)]


@dataclass
class QuestionBatch:
    index: list[int]        # positions of the batch's rows among the request's pieces
    ids: torch.Tensor       # [rows, width] int64 on the device, right-padded with pad_id
    lengths: list[int]      # tokens per row (host), as the stack's questions() takes them
    lengths_dev: torch.Tensor  # the same lengths, int32 on the device


class QuestionBatcher:
    """Builds a request's question batches on ``device`` (see the module docstring).

    ``batches(pieces, batch_size)`` yields one ``QuestionBatch`` per batch in the
    reference's order. Host staging is pinned when the device is a GPU."""

    def __init__(self, device: torch.device | str, pad_id: int, *, stream: torch.cuda.Stream | None = None):
        self.device = torch.device(device)
        self.pad_id = int(pad_id)
        self.stream = stream
        self._cuda = self.device.type == "cuda"
        self._staging: list[torch.Tensor | None] = [None, None]
        self._done: list[torch.cuda.Event | None] = [None, None]
        self._turn = 0

    def _buffer(self, nbytes: int) -> tuple[int, torch.Tensor]:
        slot = self._turn
        self._turn ^= 1
        if self._done[slot] is not None:
            self._done[slot].synchronize()  # the copy that last read this buffer has finished
        buf = self._staging[slot]
        if buf is None or buf.numel() < nbytes:
            cap = max(nbytes, 1 << 16)
            buf = torch.empty(cap, dtype=torch.uint8, pin_memory=self._cuda)
            self._staging[slot] = buf
        return slot, buf

    def build(self, rows: Sequence[Sequence[int]]) -> tuple[torch.Tensor, torch.Tensor]:
        """Padded ids ``[len(rows), max len]`` int64 and lengths int32, on the device."""
        n = len(rows)
        width = max((len(r) for r in rows), default=0)
        id_bytes = n * width * 8
        nbytes = id_bytes + n * 4
        slot, buf = self._buffer(nbytes)
        host = buf[:nbytes].numpy()
        ids = host[:id_bytes].view(np.int64).reshape(n, width)
        ids.fill(self.pad_id)
        lens = host[id_bytes:nbytes].view(np.int32)
        for r, piece in enumerate(rows):
            k = len(piece)
            lens[r] = k
            if k:
                ids[r, :k] = piece
        stream = self.stream if self.stream is not None else (
            torch.cuda.current_stream(self.device) if self._cuda else None)
        if self._cuda:
            with torch.cuda.stream(stream):
                dev = buf[:nbytes].to(self.device, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
            self._done[slot] = ev
        else:
            dev = buf[:nbytes].clone()
        ids_dev = dev[:id_bytes].view(torch.int64).view(n, width)
        lens_dev = dev[id_bytes:nbytes].view(torch.int32)
        return ids_dev, lens_dev

    def batches(self, pieces: Sequence[Sequence[int]], batch_size: int) -> Iterator[QuestionBatch]:
        for index in batch_orders(pieces, batch_size):
            rows = [pieces[i] for i in index]
            ids, lens_dev = self.build(rows)
            yield QuestionBatch(index=index, ids=ids, lengths=[len(r) for r in rows], lengths_dev=lens_dev)
