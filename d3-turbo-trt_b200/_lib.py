"""ctypes binding of libd3b200.so (the C ABI declared in include/d3b200.h).

There is no fallback: if the library is missing or a call fails, a
``RuntimeError`` names the status. Every call enqueues on the caller's current
CUDA stream of the tensor's device.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path
from typing import Any

import torch

LIB_PATH = Path(__file__).resolve().parent / "libd3b200.so"

OK, EINVAL, EALIGN, EUNSUPPORTED, ECUDA, ETIMEOUT, ENOSPACE = 0, -1, -2, -3, -4, -5, -6
F32, F16, BF16, I32 = 0, 1, 2, 3
MODE_FP8, MODE_INT8, MODE_NONE = 0, 1, 2

# (name, restype, argtypes) for every symbol include/d3b200.h declares.
_VP, _I, _I64, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
_I64P = ctypes.POINTER(ctypes.c_int64)
_U64, _U64P = ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)


class CopySegment(ctypes.Structure):
    """``d3b_copy_segment``: outer x rows rows of row_bytes bytes, byte strides on both sides."""

    _fields_ = [
        ("src", ctypes.c_void_p),
        ("dst", ctypes.c_void_p),
        ("outer", ctypes.c_int64),
        ("rows", ctypes.c_int64),
        ("row_bytes", ctypes.c_int64),
        ("src_outer_stride", ctypes.c_int64),
        ("src_row_stride", ctypes.c_int64),
        ("dst_outer_stride", ctypes.c_int64),
        ("dst_row_stride", ctypes.c_int64),
    ]


SIGNATURES: list[tuple[str, Any, list[Any]]] = [
    ("d3b_version", _I, []),
    ("d3b_error_string", ctypes.c_char_p, [_I]),
    ("d3b_device_error", _I, [_VP, _I]),
    ("d3b_act_quant", _I, [_VP, _I, _I64, _VP, _VP, _I64, _I64, _I, _VP]),
    (
        "d3b_add_rmsnorm_quant",
        _I,
        [_VP, _I64, _VP, _I64, _VP, _F, _VP, _VP, _I64, _VP, _I64, _VP, _VP, _I64, _I64, _I, _VP],
    ),
    ("d3b_sigmoid_gate_quant", _I, [_VP, _I64P, _VP, _I64P, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP]),
    ("d3b_w8a8_gemm", _I, [_VP, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _I, _I, _VP]),
    (
        "d3b_prefix_bidir",
        _I,
        [_VP, _I64P, _VP, _VP, _I64P, _VP, _VP, _I64P, _VP, _I, _I, _I, _I, _I, _I, _I, _F, _VP, _I64P, _VP],
    ),
    (
        "d3b_prefix_bidir_ws",
        _I,
        [_VP, _I64P, _VP, _VP, _I64P, _VP, _VP, _I64P, _VP, _I, _I, _I, _I, _I, _I, _I, _F, _VP, _I64P, _VP, _SZ,
         _VP],
    ),
    ("d3b_prefix_bidir_workspace_size", _SZ, [_I, _I, _I, _I, _I, _I]),
    ("d3b_causal_conv1d_silu", _I, [_VP, _I64P, _VP, _I64P, _VP, _VP, _I, _I, _I, _I, _VP]),
    ("d3b_silu_mul_quant", _I, [_VP, _I64, _VP, _VP, _VP, _I64, _I64, _I, _VP]),
    ("d3b_gated_rmsnorm_quant", _I, [_VP, _I64, _VP, _I64, _VP, _F, _I, _VP, _VP, _VP, _I64, _I64, _I, _VP]),
    ("d3b_qk_norm_rope", _I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _F, _VP]),
    ("d3b_gdn_gates", _I, [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _I, _VP]),
    ("d3b_readout_workspace_size", _SZ, [_I, _I]),
    ("d3b_readout", _I, [_VP, _I, _VP, _VP, _F, _VP, _I, _I, _I, _VP, _SZ, _VP]),
    ("d3b_readout_noalloc", _I, [_VP, _I, _VP, _VP, _F, _VP, _I, _I, _I, _VP]),
    ("d3b_readout_planes_size", _SZ, [_I, _I]),
    ("d3b_readout_split", _I, [_VP, _I, _I, _VP, _VP]),
    ("d3b_readout_planes_workspace_size", _SZ, [_I, _I, _I]),
    ("d3b_readout_planes", _I, [_VP, _VP, _VP, _F, _VP, _I, _I, _I, _VP, _SZ, _VP]),
    ("d3b_selftest_wait_timeout", _I, [_I, _VP]),
    (
        "d3b_gated_delta_rule",
        _I,
        [_VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _I64P, _VP, _I, _I64P, _VP, _I64P, _VP, _I64P, _VP,
         _I, _I, _I, _I, _I, _I, _I, _F, _I, _I, _VP, _SZ, _VP],
    ),
    ("d3b_gated_delta_workspace_size", _SZ, [_I, _I, _I]),
    ("d3b_gated_delta_state_workspace_size", _SZ, [_I, _I, _I, _I, _I]),
    ("d3b_copy_segments", _I, [ctypes.POINTER(CopySegment), _I, _VP]),
    ("d3b_arena_create", _I, [_U64, _U64, ctypes.POINTER(ctypes.c_void_p)]),
    ("d3b_arena_alloc", _I, [_VP, _U64, _U64P]),
    ("d3b_arena_free", _I, [_VP, _U64]),
    ("d3b_arena_stats", _I, [_VP, _U64P]),
    ("d3b_arena_destroy", None, [_VP]),
]

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libd3b200.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built (expected at {LIB_PATH}); "
                    "run `python d3-turbo-trt_b200/csrc/build.py` or __graft_entry__.build()"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, restype, argtypes in SIGNATURES:
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def error_string(status: int) -> str:
    return lib().d3b_error_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != OK:
        raise RuntimeError(f"{what}: libd3b200 status {status} ({error_string(status)})")


def stream_of(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def i64_array(values) -> Any:
    arr = (ctypes.c_int64 * len(values))(*[int(v) for v in values])
    return arr


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float16:
        return F16
    if dtype == torch.float32:
        return F32
    if dtype == torch.int32:
        return I32
    raise RuntimeError(f"unsupported dtype {dtype}")


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} needs CUDA tensors (the CPU formulas live in the test oracle only)")
    lib()


_ERROR_RESET_HOOKS: list = []


def on_device_error(hook) -> None:
    """Register ``hook(device_index)``, called when ``device_error`` reads a
    non-zero word with ``reset``: state that a launch which gave up may have
    left behind (a workspace's counters) is restored there."""
    _ERROR_RESET_HOOKS.append(hook)


def device_error(device: torch.device | int | None = None, reset: bool = True) -> int:
    """Device error word after synchronising the current stream (0 = none).

    The word is sticky: once a device-side wait has given up, later launches
    stop early and their outputs are undefined until it is read with
    ``reset``; check it after a pass (or a batch of passes)."""
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if dev.index is None:  # plain "cuda": the current device, as torch resolves it
            dev = torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        word = int(lib().d3b_device_error(s, 1 if reset else 0))
        if word and reset:
            for hook in _ERROR_RESET_HOOKS:
                hook(dev.index)
        return word
