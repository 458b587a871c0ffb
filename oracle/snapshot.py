"""Packed-snapshot oracle (numpy) — test infrastructure only.

Restates the packing rule of the state-cache format: every tensor of a snapshot
(the per-layer entries of d3trt/model/core.py:28-40, walked entry by entry and
field by field) is stored dense, with its dimensions ordered like the source's
strides (outermost = largest stride; equal strides keep index order), at the
next 256-byte boundary after the previous tensor. Packing is a byte copy, so
parity is bit-exact.

Also an interpreter of ``d3b_copy_segments`` semantics over flat byte arrays,
used to check the host-side piece planner on the CPU.
"""

from __future__ import annotations

import numpy as np
import torch

ALIGNMENT = 256


def dense_in_stride_order(t) -> np.ndarray:
    """A torch tensor's elements, as raw bytes, laid out dense in its stride order."""
    if t.numel() == 0:
        return np.zeros(0, np.uint8)
    shape, strides = list(t.shape), list(t.stride())
    order = sorted((i for i in range(len(shape)) if shape[i] > 1), key=lambda i: (-strides[i], i))
    rest = [i for i in range(len(shape)) if i not in order]
    arr = t.detach().cpu().contiguous()
    elems = arr.view(-1).view(torch.uint8).numpy().reshape(*arr.shape, arr.element_size())
    return np.ascontiguousarray(elems.transpose(rest + order + [len(shape)])).reshape(-1)


def pack(tensors) -> tuple[list[tuple[int, np.ndarray]], int]:
    """([(offset, bytes)] per tensor, block bytes) for a flat list of tensors; None takes no space."""
    placed, off = [], 0
    for t in tensors:
        if t is None:
            placed.append((off, np.zeros(0, np.uint8)))
            continue
        b = dense_in_stride_order(t)
        placed.append((off, b))
        off += len(b) + (-len(b) % ALIGNMENT)
    return placed, max(off, ALIGNMENT)


def apply_segments(src: np.ndarray, dst: np.ndarray, segments) -> None:
    """Run copy segments (src_off, dst_off, outer, rows, row_bytes, s_outer, s_row, d_outer, d_row), byte units."""
    for so, do, outer, rows, row_bytes, s_o, s_r, d_o, d_r in segments:
        for o in range(outer):
            for r in range(rows):
                a = so + o * s_o + r * s_r
                b = do + o * d_o + r * d_r
                dst[b:b + row_bytes] = src[a:a + row_bytes]
