"""Shared-prefix bidirectional attention on sm_100a (drop-in for d3trt/kernels/prefix_bidir.py).

``prefix_bidir_attention(q, k_state, v_state, k_q, v_q, lengths, *, scale)``
keeps the reference signature and layouts (prefix_bidir.py:187-260):

    q        [B, H, L, D]   right-padded question blocks (any strides, D contiguous)
    k_state  [H_kv, S, D]   shared state prefix, RoPE applied (head- or token-major)
    v_state  [H_kv, S, D]
    k_q, v_q [B, H_kv, L, D]
    lengths  real tokens per block (Python ints or an int tensor)
    returns  [B, H, L, D], zero rows for padding

It launches one tcgen05/TMA kernel (libd3b200 ``d3b_prefix_bidir``): no
pack/unpack gathers (reference :225-231, :260) and no token-major copies of the
state K/V (:179-184) — the TMA descriptors read any 16-byte-multiple strides.
``state_attention`` is the dense bidirectional state pass over the same kernel
(drop-in for ``ops.flash_state`` / ``ops.sdpa_state``).

Error behaviour follows the reference: ``RuntimeError`` for a CPU tensor, a
dtype other than fp16/bf16, mixed dtypes, an unsupported head_dim or heads not
divisible by kv heads (prefix_bidir.py:202-216). There is no fallback.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Sequence

import torch

from .. import _lib

HEAD_DIMS = (32, 64, 128, 256)
KERNEL_NAME = "sm100a"
# Device error word set by the kernel when a device-resident lengths entry lies
# outside [0, L] (the entry is clamped; read it with _lib.device_error()).
SITE_BAD_LENGTH = 2010

_LENGTHS: "OrderedDict[tuple, torch.Tensor]" = OrderedDict()
_LENGTHS_MAX = 16

# Workspaces of d3b_prefix_bidir_ws, one per (device, stream): zero-filled when
# made; every launch leaves them zeroed again and calls on one stream are
# ordered, so they are reused as they are.
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, torch.cuda.current_stream(index).cuda_stream)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", index))
        _WORKSPACES[key] = buf
    return buf


def _rezero_workspaces(index: int) -> None:
    # a launch that gave up may have left a unit's count behind
    for (dev, _), buf in _WORKSPACES.items():
        if dev == index:
            buf.zero_()


_lib.on_device_error(_rezero_workspaces)


def kernel_available() -> bool:
    """True when libd3b200 is built and a CUDA device is present."""
    try:
        _lib.lib()
    except RuntimeError:
        return False
    return torch.cuda.is_available()


def triton_available() -> bool:  # name kept for callers of the reference module
    return kernel_available()


def block_offsets(lengths: Sequence[int] | torch.Tensor, device: torch.device) -> torch.Tensor:
    """The block-offset table as a device int32 tensor of lengths, cached like the
    reference ``_meta`` (prefix_bidir.py:152-163, an LRU of 16 by (lengths, device))."""
    if isinstance(lengths, torch.Tensor):
        if lengths.is_cuda and lengths.dtype == torch.int32 and lengths.device == device:
            return lengths.contiguous()
        lengths = [int(n) for n in lengths.tolist()]
    key = (tuple(int(n) for n in lengths), str(device))
    hit = _LENGTHS.get(key)
    if hit is not None:
        _LENGTHS.move_to_end(key)
        return hit
    if len(_LENGTHS) >= _LENGTHS_MAX:
        _LENGTHS.popitem(last=False)
    t = torch.tensor(key[0], dtype=torch.int32).to(device, non_blocking=False)
    _LENGTHS[key] = t
    return t


def _check(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    if not q.is_cuda:
        raise RuntimeError("the prefix-bidir kernel needs CUDA")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("the prefix-bidir kernel needs fp16 or bf16")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise RuntimeError("q, k and v must share a dtype")
    if q.shape[-1] not in HEAD_DIMS:
        raise RuntimeError(f"unsupported head_dim {q.shape[-1]}")


def _inner_contig(x: torch.Tensor) -> torch.Tensor:
    """Keep any strides except a non-unit last stride or a misaligned view."""
    if x.stride(-1) != 1 or x.data_ptr() % 16 or any(s % 8 for s in x.stride()[:-1]):
        return x.contiguous()
    return x


def _launch(
    q: torch.Tensor,
    k_state: torch.Tensor | None,
    v_state: torch.Tensor | None,
    k_q: torch.Tensor,
    v_q: torch.Tensor,
    lens: torch.Tensor,
    scale: float,
    out: torch.Tensor,
) -> None:
    rows, heads, width, dim = q.shape
    kv_heads = k_q.shape[1]
    state = 0 if k_state is None else int(k_state.shape[1])
    if state == 0:
        k_state = v_state = None
    st_q = _lib.i64_array(q.stride()[:3])
    st_kq = _lib.i64_array(k_q.stride()[:3])
    st_out = _lib.i64_array(out.stride()[:3])
    st_kv = _lib.i64_array(k_state.stride()[:2]) if k_state is not None else None
    if k_state is not None and (k_state.stride() != v_state.stride()):
        raise RuntimeError("k_state and v_state must share strides")
    if k_q.stride() != v_q.stride():
        raise RuntimeError("k_q and v_q must share strides")
    lib = _lib.lib()
    ws = _workspace(q.device, int(lib.d3b_prefix_bidir_workspace_size(rows, heads, kv_heads, state, width, dim)))
    status = lib.d3b_prefix_bidir_ws(
        _lib.ptr(q), st_q, _lib.ptr(k_state), _lib.ptr(v_state), st_kv, _lib.ptr(k_q), _lib.ptr(v_q), st_kq,
        _lib.ptr(lens), rows, heads, kv_heads, state, width, dim, _lib.dtype_code(q.dtype), float(scale),
        _lib.ptr(out), st_out, _lib.ptr(ws), 0 if ws is None else ws.numel(), _lib.stream_of(q),
    )
    _lib.check(status, "d3b_prefix_bidir_ws")


def prefix_bidir_attention(
    q: torch.Tensor,
    k_state: torch.Tensor,
    v_state: torch.Tensor,
    k_q: torch.Tensor,
    v_q: torch.Tensor,
    lengths: Sequence[int] | torch.Tensor,
    *,
    scale: float,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Bidirectional question attention over a shared state prefix (prefix_bidir.py:187-260).

    Inputs follow the model's natural layout: q/k_q/v_q are [B, H, L, D],
    k_state/v_state are [H_kv, S, D]. Returns [B, H, L, D]. ``out`` may be a
    preallocated [B, H, L, D] tensor (any strides, D contiguous).

    ``lengths`` given as Python ints are checked here (``RuntimeError`` outside
    [0, L]). A CUDA int32 tensor is passed to the kernel as it is, without a
    device sync; the kernel clamps entries outside [0, L] and sets the device
    error word to ``SITE_BAD_LENGTH``, which ``_lib.device_error()`` returns.
    """
    _check(q, k_q, v_q)
    if k_state.dtype != q.dtype or v_state.dtype != q.dtype:
        raise RuntimeError("q, k and v must share a dtype")
    rows, heads, width, dim = q.shape
    kv_heads = k_state.shape[0]
    if heads % kv_heads:
        raise RuntimeError("heads must be divisible by kv heads")
    if tuple(k_q.shape) != (rows, kv_heads, width, dim) or tuple(v_q.shape) != tuple(k_q.shape):
        raise RuntimeError(f"k_q/v_q must be [B, H_kv, L, D] = {(rows, kv_heads, width, dim)}")
    if tuple(v_state.shape) != tuple(k_state.shape) or k_state.shape[2] != dim:
        raise RuntimeError("k_state/v_state must be [H_kv, S, D]")
    _lib.lib()
    if out is None:
        out = torch.empty((rows, heads, width, dim), dtype=q.dtype, device=q.device)
    if isinstance(lengths, torch.Tensor):
        n_rows = lengths.numel()
    else:
        lengths = [int(n) for n in lengths]
        n_rows = len(lengths)
        if lengths and (max(lengths) > width or min(lengths) < 0):
            raise RuntimeError(f"lengths must lie in [0, {width}]")
        if sum(lengths) == 0 and n_rows == rows:
            out.zero_()
            return out
    if n_rows != rows:
        raise RuntimeError(f"{n_rows} lengths for {rows} question blocks")
    if rows == 0 or width == 0:
        return out
    lens = block_offsets(lengths, q.device)
    _launch(
        _inner_contig(q), _inner_contig(k_state), _inner_contig(v_state), _inner_contig(k_q), _inner_contig(v_q),
        lens, scale, out,
    )
    return out


def state_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense bidirectional attention of the state block over itself, [B, H, S, D].

    Drop-in for ``ops.flash_state`` / ``ops.sdpa_state`` (ops.py:107-124, :174-193):
    q [B, H, S, D], k/v [B, H_kv, S, D], GQA native, no transposes or copies.
    ``out`` may be a preallocated [B, H, S, D] tensor (any strides, D contiguous).
    """
    _check(q, k, v)
    rows, heads, tokens, dim = q.shape
    if heads % k.shape[1]:
        raise RuntimeError("heads must be divisible by kv heads")
    if tuple(k.shape) != (rows, k.shape[1], tokens, dim) or tuple(v.shape) != tuple(k.shape):
        raise RuntimeError("k/v must be [B, H_kv, S, D] matching q")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    elif tuple(out.shape) != tuple(q.shape) or out.dtype != q.dtype or out.stride(-1) != 1:
        raise RuntimeError("out must be [B, H, S, D] like q with a contiguous last dimension")
    if rows == 0 or tokens == 0:
        return out
    lens = block_offsets([tokens] * rows, q.device)
    _launch(_inner_contig(q), None, None, _inner_contig(k), _inner_contig(v), lens, scale, out)
    return out
