"""255-way fp32 readout softmax on sm_100a (drop-in for the ``probabilities`` method of
d3trt/model/trtllm_stack.py:451-468, identical to hf_stack.py:67-84).

    logits = hidden.float() @ readout.T
    logits[b, j >= counts[b]] = -inf
    probs  = softmax(logits / temperature)
    return [row[:count] for row, count in zip(probs.tolist(), counts)]

For bf16 hidden rows (the model's final-norm output) the dot products run on the
tensor cores: the fp32 readout matrix is split once into three bf16 planes that
carry all of its 24 bits (``d3b_readout_split``, cached per readout tensor), every
product of a bf16 hidden value with a plane value is exact in fp32, and the
planes' products accumulate in fp32 (``d3b_readout_planes``): an fp32 dot product
that differs from the reference's only in summation order. Other hidden dtypes
take the fp32 FMA kernels (``d3b_readout``). Either way a second kernel adds the
K splits and applies the mask, the temperature and the softmax; the only host
work left is the device-to-host copy of the result, as in the reference
(``.cpu().tolist()``).
"""

from __future__ import annotations

import weakref
from typing import Sequence

import torch

from .. import _lib

KERNEL_NAME = "sm100a"
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}
_PARTIALS: dict[tuple[int, int], torch.Tensor] = {}  # the tensor-core path's partial logits (no zeroing needed)
_PLANES: dict[tuple, tuple] = {}  # readout matrix -> (weak ref to it, its three bf16 planes); a few recent ones


def readout_planes(readout: torch.Tensor) -> torch.Tensor:
    """The three bf16 planes of an fp32 readout matrix on its device, cached per tensor
    object, address, shape and version: an in-place change of the matrix makes new planes,
    and so does a new matrix that the allocator placed where a freed one was (the entry
    holds a weak reference to the tensor it was made from and is used only for that tensor)."""
    key = (readout.device.index, readout.data_ptr(), tuple(readout.shape), readout._version)
    entry = _PLANES.get(key)
    planes = entry[1] if entry is not None and entry[0]() is readout else None
    if planes is None:
        n_opt, k = readout.shape
        lib = _lib.lib()
        planes = torch.empty(int(lib.d3b_readout_planes_size(n_opt, k)) // 2, dtype=torch.bfloat16,
                             device=readout.device)
        with torch.cuda.device(readout.device):
            _lib.check(lib.d3b_readout_split(_lib.ptr(readout), n_opt, k, _lib.ptr(planes), _lib.stream_of(readout)),
                       "d3b_readout_split")
        _PLANES.pop(key, None)
        if len(_PLANES) >= 4:
            _PLANES.pop(next(iter(_PLANES)))
        _PLANES[key] = (weakref.ref(readout), planes)
    return planes


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """A zero-filled scratch buffer per (device, stream); calls on one stream never overlap."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def probabilities_tensor(
    hidden: torch.Tensor,
    readout: torch.Tensor,
    counts: Sequence[int] | torch.Tensor,
    *,
    temperature: float,
) -> torch.Tensor:
    """[B, K] hidden, [n_opt, K] fp32 readout -> [B, n_opt] fp32 probabilities on the device."""
    _lib.require_cuda(hidden, "probabilities")
    if hidden.dim() != 2 or readout.dim() != 2 or hidden.shape[1] != readout.shape[1]:
        raise ValueError(f"hidden {tuple(hidden.shape)} and readout {tuple(readout.shape)} do not match")
    if hidden.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        hidden = hidden.float()
    hidden = hidden.contiguous()
    readout = readout.to(device=hidden.device, dtype=torch.float32).contiguous()
    rows, k = hidden.shape
    n_opt = readout.shape[0]
    if isinstance(counts, torch.Tensor):
        counts_t = counts.to(device=hidden.device, dtype=torch.int32).contiguous()
    else:
        counts_t = torch.tensor([int(c) for c in counts], dtype=torch.int32).to(hidden.device)
    if counts_t.numel() != rows:
        raise ValueError(f"{counts_t.numel()} counts for {rows} rows")
    probs = torch.empty((rows, n_opt), dtype=torch.float32, device=hidden.device)
    if rows == 0:
        return probs
    lib = _lib.lib()
    stream = _lib.stream_of(hidden)
    if hidden.dtype == torch.bfloat16 and k % 8 == 0 and hidden.data_ptr() % 16 == 0:
        planes = readout_planes(readout)
        nbytes = int(lib.d3b_readout_planes_workspace_size(rows, k, n_opt))
        # its own buffer: d3b_readout's workspace holds ticket counters that must stay zero
        key = (hidden.device.index, int(stream.value or 0))
        ws = _PARTIALS.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=hidden.device)
            _PARTIALS[key] = ws
        status = lib.d3b_readout_planes(
            _lib.ptr(hidden), _lib.ptr(planes), _lib.ptr(counts_t), float(temperature), _lib.ptr(probs), rows, k,
            n_opt, _lib.ptr(ws), ws.numel(), stream,
        )
        _lib.check(status, "d3b_readout_planes")
        return probs
    nbytes = int(lib.d3b_readout_workspace_size(rows, n_opt))
    ws = _workspace(hidden.device, int(stream.value or 0), nbytes)
    status = lib.d3b_readout(
        _lib.ptr(hidden), _lib.dtype_code(hidden.dtype), _lib.ptr(readout), _lib.ptr(counts_t), float(temperature),
        _lib.ptr(probs), rows, k, n_opt, _lib.ptr(ws), ws.numel(), stream,
    )
    _lib.check(status, "d3b_readout")
    return probs


def probabilities(
    hidden: torch.Tensor,
    readout: torch.Tensor,
    counts: Sequence[int],
    *,
    temperature: float,
    readout_dtype: str = "float32",
) -> list[list[float]]:
    """Per-answer probabilities, rows cut to ``count`` (trtllm_stack.py:451-468)."""
    if readout_dtype != "float32":
        raise ValueError("the sm_100a readout computes in float32 only (readout_dtype='float32')")
    counts = [int(c) for c in counts]
    values = probabilities_tensor(hidden, readout, counts, temperature=temperature).cpu().tolist()
    return [row[:count] for row, count in zip(values, counts)]


class ReadoutHead:
    """The ``probabilities`` method of the reference stacks, bound to a readout matrix."""

    def __init__(self, readout: torch.Tensor):
        self.readout = readout.float().contiguous()
        self.max_options = int(readout.shape[0])

    def probabilities(
        self,
        hidden: torch.Tensor,
        counts: Sequence[int],
        *,
        temperature: float,
        readout_dtype: str = "float32",
    ) -> list[list[float]]:
        return probabilities(hidden, self.readout, counts, temperature=temperature, readout_dtype=readout_dtype)
