"""Failure detection on the GPU without a fault: a device-side wait that nothing
completes runs out of its limit, the kernel records its site code and returns,
the host reads the code, and the context stays usable."""

from __future__ import annotations

import ctypes

import pytest
import torch

from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.model import quant

pytestmark = pytest.mark.gpu


def test_wait_limit_reports_and_context_survives():
    assert _lib.device_error() == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert _lib.lib().d3b_selftest_wait_timeout(200, stream) == _lib.OK
    assert _lib.device_error(reset=True) == 9001
    assert _lib.device_error() == 0
    q, s = quant.quantize_rows(torch.ones(4, 64, device="cuda"), "int8")
    assert torch.all(q == 127)
