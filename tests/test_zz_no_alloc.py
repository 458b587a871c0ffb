"""The allocation-free readout entry point, called through the C ABI.

d3b_readout_noalloc serves callers that cannot allocate device memory when
they call (graph-capture regions, runtimes that only pass in and out
buffers): its scratch lives in a fixed array inside the library. These tests
check it against the workspace-based d3b_readout on the same inputs, on two
calls in a row (the second call finds the first call's leftovers in the shared
array), and that a request beyond the array's 1 MiB is refused up front.

This file is collected last on purpose, so a run that stops at its first
failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from d3_turbo_trt_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-5  # the readout tests' tolerance


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(hidden, readout, counts, temperature, probs) -> int:
    lib = _lib.lib()
    rows, k = hidden.shape
    n_opt = readout.shape[0]
    nbytes = int(lib.d3b_readout_workspace_size(rows, n_opt))
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    return lib.d3b_readout(_ptr(hidden), _lib.BF16, _ptr(readout), _ptr(counts), float(temperature), _ptr(probs),
                           rows, k, n_opt, _ptr(ws), nbytes, _stream())


def _no_alloc(hidden, readout, counts, temperature, probs) -> int:
    rows, k = hidden.shape
    return _lib.lib().d3b_readout_noalloc(_ptr(hidden), _lib.BF16, _ptr(readout), _ptr(counts), float(temperature),
                                          _ptr(probs), rows, k, readout.shape[0], _stream())


def _inputs(seed: int, rows: int, k: int, n_opt: int):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(rows, k, generator=g).to(torch.bfloat16).to(DEV)
    readout = (torch.randn(n_opt, k, generator=g) * 0.02).to(DEV)
    counts = torch.tensor([1 + (i * 37 + seed) % n_opt for i in range(rows)], dtype=torch.int32, device=DEV)
    return hidden, readout, counts


def test_no_alloc_matches_workspace_readout_twice():
    # two calls in a row, different shapes and temperatures
    for seed, (rows, k, n_opt, temp) in enumerate(((255, 5120, 255, 1.0), (97, 1024, 255, 0.7))):
        hidden, readout, counts = _inputs(seed, rows, k, n_opt)
        want = torch.full((rows, n_opt), -1.0, device=DEV)
        got = torch.full((rows, n_opt), -2.0, device=DEV)
        assert _with_workspace(hidden, readout, counts, temp, want) == _lib.OK
        assert _no_alloc(hidden, readout, counts, temp, got) == _lib.OK
        torch.cuda.synchronize()
        w, g_ = want.cpu().numpy(), got.cpu().numpy()
        assert np.abs(w - g_).max() <= TOL
        assert np.allclose(g_.sum(axis=1), 1.0, atol=1e-4)
    assert _lib.device_error() == 0


def test_no_alloc_refuses_requests_beyond_its_array():
    hidden, readout, counts = _inputs(3, 8, 64, 255)
    probs = torch.empty(8, 255, device=DEV)
    lib = _lib.lib()
    # 1100 x 255 logits need more than 1 MiB: refused before any launch
    assert lib.d3b_readout_noalloc(_ptr(hidden), _lib.BF16, _ptr(readout), _ptr(counts), 1.0, _ptr(probs), 1100, 64,
                                   255, _stream()) == _lib.ENOSPACE
    # the array still serves a valid call afterwards
    assert _no_alloc(hidden, readout, counts, 1.0, probs) == _lib.OK
    torch.cuda.synchronize()
    assert torch.isfinite(probs).all()
