"""The C-ABI boundary without a GPU: the library loads, exports exactly what
include/d3b200.h declares, and rejects bad arguments on the host (before any
CUDA call). Also the Python wrappers' reference-compatible error behaviour
(d3trt/kernels/prefix_bidir.py:202-216, d3trt/model/quant.py:116-143)."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest
import torch

from conftest import ROOT

import d3_turbo_trt_b200 as d3b
from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.kernels import prefix_bidir as pb
from d3_turbo_trt_b200.model import ops, quant

HEADER = ROOT / "include" / "d3b200.h"


def header_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"D3B_API\s+[\w\s\*]+?\b(d3b_\w+)\s*\(", text))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = header_symbols()
    assert declared == {name for name, _, _ in _lib.SIGNATURES}
    for name in declared:
        assert getattr(lib, name) is not None
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\b(d3b_\w+)\b", out.stdout))
    assert declared <= exported
    assert lib.d3b_version() == 100


def test_error_strings():
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert _lib.error_string(code) != "unknown status"
    assert _lib.error_string(-99) == "unknown status"


def test_act_quant_rejects_bad_arguments():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)
    assert lib.d3b_act_quant(p, _lib.BF16, 8, p, p, 4, 8, 7, None) == _lib.EINVAL  # bad mode
    assert lib.d3b_act_quant(p, _lib.BF16, 4, p, p, 4, 8, 0, None) == _lib.EINVAL  # ldx < K
    assert lib.d3b_act_quant(p, _lib.BF16, 8, p, p, -1, 8, 0, None) == _lib.EINVAL
    assert lib.d3b_act_quant(p, 9, 8, p, p, 4, 8, 0, None) == _lib.EUNSUPPORTED
    assert lib.d3b_act_quant(p, _lib.BF16, 8, p, p, 0, 8, 0, None) == _lib.OK  # empty is a no-op


def test_gemm_rejects_bad_arguments():
    lib = _lib.lib()
    a = ctypes.c_void_p(256)
    assert lib.d3b_w8a8_gemm(a, a, a, a, a, 32, 16, 32, 24, 0, _lib.BF16, None) == _lib.EINVAL  # K % 16
    assert lib.d3b_w8a8_gemm(a, a, a, a, a, 40, 16, 40, 32, 0, _lib.BF16, None) == _lib.EINVAL  # N % 16
    assert lib.d3b_w8a8_gemm(a, a, a, a, a, 32, 16, 32, 32, 0, _lib.I32, None) == _lib.EUNSUPPORTED  # raw i32 is int8-only
    assert lib.d3b_w8a8_gemm(a, a, a, a, ctypes.c_void_p(258), 32, 16, 32, 32, 0, _lib.BF16, None) == _lib.EALIGN
    assert lib.d3b_w8a8_gemm(a, a, a, a, a, 16, 16, 32, 32, 0, _lib.BF16, None) == _lib.EINVAL  # ldy < N
    assert lib.d3b_w8a8_gemm(a, a, a, a, a, 32, 0, 32, 32, 0, _lib.BF16, None) == _lib.OK  # M == 0


def _attn_call(**over):
    lib = _lib.lib()
    a = ctypes.c_void_p(1024)
    st = _lib.i64_array([64 * 8 * 128, 64 * 128, 128])
    kv = _lib.i64_array([64 * 128, 128])
    args = dict(q=a, qs=st, ks=a, vs=a, kvs=kv, kq=a, vq=a, kqs=st, lens=a, B=2, H=8, Hkv=2, S=64, L=8, D=128,
                dtype=_lib.BF16, scale=0.1, out=a, outs=st)
    args.update(over)
    return lib.d3b_prefix_bidir(args["q"], args["qs"], args["ks"], args["vs"], args["kvs"], args["kq"], args["vq"],
                                args["kqs"], args["lens"], args["B"], args["H"], args["Hkv"], args["S"], args["L"],
                                args["D"], args["dtype"], args["scale"], args["out"], args["outs"], None)


def test_prefix_bidir_rejects_bad_arguments():
    assert _attn_call(D=48) == _lib.EUNSUPPORTED
    assert _attn_call(H=6, Hkv=4) == _lib.EINVAL
    assert _attn_call(dtype=_lib.F32) == _lib.EUNSUPPORTED
    assert _attn_call(H=256, Hkv=1) == _lib.EUNSUPPORTED  # group > 128 rows
    assert _attn_call(scale=-1.0) == _lib.EINVAL
    assert _attn_call(q=ctypes.c_void_p(1026)) == _lib.EALIGN
    assert _attn_call(qs=_lib.i64_array([64 * 8 * 128, 64 * 128, 130])) == _lib.EALIGN
    assert _attn_call(B=0) == _lib.OK
    assert _attn_call(L=0) == _lib.OK


def test_readout_rejects_bad_arguments():
    lib = _lib.lib()
    a = ctypes.c_void_p(256)
    need = lib.d3b_readout_workspace_size(255, 255)
    assert need >= 255 * 255 * 4
    assert lib.d3b_readout(a, _lib.BF16, a, a, 1.0, a, 255, 64, 255, a, need - 1, None) == _lib.ENOSPACE
    assert lib.d3b_readout(a, _lib.BF16, a, a, 0.0, a, 255, 64, 255, a, need, None) == _lib.EINVAL
    assert lib.d3b_readout(a, _lib.BF16, a, a, 1.0, a, 4, 64, 2000, a, need, None) == _lib.EINVAL
    assert lib.d3b_readout(a, 7, a, a, 1.0, a, 4, 64, 255, a, need, None) == _lib.EUNSUPPORTED
    assert lib.d3b_readout_workspace_size(0, 255) == 0
    assert lib.d3b_readout(a, _lib.BF16, a, a, 1.0, a, 8 * 4096 + 1, 64, 255, a, 1 << 40, None) == _lib.EINVAL


def test_readout_planes_rejects_bad_arguments():
    lib = _lib.lib()
    a = ctypes.c_void_p(256)
    assert lib.d3b_readout_planes_size(255, 5120) == 3 * 256 * 5120 * 2
    assert lib.d3b_readout_planes_size(257, 64) == 3 * 512 * 64 * 2
    need = lib.d3b_readout_planes_workspace_size(255, 5120, 255)
    assert need >= 256 * 256 * 4  # at least one split of padded partial logits
    assert lib.d3b_readout_planes(a, a, a, 1.0, a, 255, 5120, 255, a, need - 1, None) == _lib.ENOSPACE
    assert lib.d3b_readout_planes(a, a, a, 0.0, a, 255, 5120, 255, a, need, None) == _lib.EINVAL
    assert lib.d3b_readout_planes(a, a, a, 1.0, a, 4, 64, 2000, a, need, None) == _lib.EINVAL
    assert lib.d3b_readout_planes(a, a, a, 1.0, a, 4, 100, 255, a, 1 << 30, None) == _lib.EUNSUPPORTED  # K % 8
    assert lib.d3b_readout_planes(ctypes.c_void_p(258), a, a, 1.0, a, 4, 64, 255, a, 1 << 30, None) == _lib.EALIGN
    assert lib.d3b_readout_planes(a, a, a, 1.0, a, 0, 64, 255, a, 0, None) == _lib.OK  # no rows: nothing to do
    assert lib.d3b_readout_split(None, 255, 64, a, None) == _lib.EINVAL
    assert lib.d3b_readout_split(a, 0, 64, a, None) == _lib.EINVAL


def test_copy_segments_rejects_bad_arguments():
    lib = _lib.lib()
    seg = _lib.CopySegment
    p = 4096
    one = (seg * 1)(seg(p, p * 2, 1, -1, 16, 0, 0, 0, 0))
    assert lib.d3b_copy_segments(one, 1, None) == _lib.EINVAL  # negative rows
    one = (seg * 1)(seg(None, p, 1, 1, 16, 0, 0, 0, 0))
    assert lib.d3b_copy_segments(one, 1, None) == _lib.EINVAL  # null source with bytes to move
    one = (seg * 1)(seg(p, p * 2, 1 << 31, 1, 16, 0, 0, 0, 0))
    assert lib.d3b_copy_segments(one, 1, None) == _lib.EINVAL  # outer count past 2^31 - 1
    assert lib.d3b_copy_segments(None, -1, None) == _lib.EINVAL
    assert lib.d3b_copy_segments(None, 0, None) == _lib.OK  # nothing to copy: no launch
    empty = (seg * 2)(seg(None, None, 0, 1, 16, 0, 0, 0, 0), seg(p, p, 3, 4, 0, 0, 0, 0, 0))
    assert lib.d3b_copy_segments(empty, 2, None) == _lib.OK  # empty segments are skipped


def test_gated_delta_rejects_bad_arguments():
    lib = _lib.lib()
    p = ctypes.c_void_p(256)
    st = _lib.i64_array([1024, 128, 64])

    def call(B=2, T=3, H=1, HV=2, K=64, V=64, dtype=_lib.BF16, beta_dtype=_lib.BF16, ptr=p, strides=st, algo=0):
        return lib.d3b_gated_delta_rule(ptr, strides, ptr, strides, ptr, strides, ptr, strides, ptr, beta_dtype,
                                        strides, None, None, ptr, strides, None, B, T, H, HV, K, V, dtype, 0.125,
                                        1, algo, None, 0, None)

    assert call(K=96) == _lib.EUNSUPPORTED
    assert call(V=48) == _lib.EINVAL
    assert call(HV=3, H=2) == _lib.EINVAL
    assert call(dtype=_lib.F32) == _lib.EUNSUPPORTED
    assert call(beta_dtype=_lib.I32) == _lib.EUNSUPPORTED
    assert call(strides=None) == _lib.EINVAL
    assert call(ptr=ctypes.c_void_p(257)) == _lib.EALIGN
    assert call(B=0) == _lib.OK  # nothing to do: no launch
    assert call(algo=4) == _lib.EINVAL
    assert call(algo=2) == _lib.EUNSUPPORTED  # the chunked form needs K = V = 128
    assert call(algo=2, K=128, V=128, T=65) == _lib.EUNSUPPORTED  # and blocks of <= 64 tokens
    assert call(algo=3) == _lib.EUNSUPPORTED  # the inter-chunk form needs K = V = 128
    assert call(algo=3, K=128, V=128) == _lib.EUNSUPPORTED  # and a workspace
    assert lib.d3b_gated_delta_workspace_size(48, 128, 128) == 48 * 32768
    assert lib.d3b_gated_delta_workspace_size(48, 64, 64) == 0
    assert lib.d3b_gated_delta_state_workspace_size(1, 4096, 48, 128, 128) == 48 * 64 * 74752
    assert lib.d3b_gated_delta_state_workspace_size(2, 65, 3, 128, 128) == 2 * 3 * 2 * 74752
    assert lib.d3b_gated_delta_state_workspace_size(1, 4096, 48, 64, 64) == 0


def test_wait_selftest_rejects_bad_limit():
    assert _lib.lib().d3b_selftest_wait_timeout(0, None) == _lib.EINVAL
    assert _lib.lib().d3b_selftest_wait_timeout(10_000, None) == _lib.EINVAL


# --- Python wrappers: reference-compatible errors, no CPU fallback ---


def test_attention_wrapper_needs_cuda():
    q = torch.zeros(1, 2, 4, 32, dtype=torch.bfloat16)
    ks = torch.zeros(1, 8, 32, dtype=torch.bfloat16)
    kq = torch.zeros(1, 1, 4, 32, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="needs CUDA"):
        pb.prefix_bidir_attention(q, ks, ks, kq, kq, [4], scale=0.1)
    with pytest.raises(RuntimeError, match="needs CUDA"):
        ops.question_attention(q, ks, ks, kq, kq, [4], scale=0.1)
    with pytest.raises(RuntimeError, match="needs CUDA"):
        ops.flash_state(q, kq, kq, scale=0.1)


def test_quant_wrappers_need_cuda():
    with pytest.raises(RuntimeError, match="CUDA"):
        quant.quantize_rows(torch.randn(4, 32), "fp8")
    layer = quant.QuantLinear(64, 32, mode="int8", dtype=torch.float32, device="cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        layer.load_full(torch.randn(32, 64))
    with pytest.raises(RuntimeError, match="CUDA"):
        d3b.probabilities(torch.randn(2, 16), torch.randn(4, 16), [4, 4], temperature=1.0)


def test_shape_checks():  # reference tests/test_quant.py:53-60
    assert quant.quantizable(5120, 17408)
    assert not quant.quantizable(5120, 40)
    with pytest.raises(ValueError):
        quant.QuantLinear(64, 40, mode="fp8", dtype=torch.bfloat16, device="cpu")
    layer = quant.QuantLinear(64, 32, mode="fp8", dtype=torch.bfloat16, device="cpu")
    with pytest.raises(ValueError):
        layer.load_full(torch.zeros(32, 48))
    with pytest.raises(ValueError):
        quant.QuantLinear(64, 32, mode="none", dtype=torch.bfloat16, device="cpu")


def test_resolve_mode_off_gpu():  # reference tests/test_quant.py:63-68
    assert quant.resolve_mode("auto", "cpu") == "none"
    assert quant.resolve_mode("int8", "cpu") == "int8"
    assert quant.resolve_mode("fp8", "cpu") == "fp8"
    with pytest.raises(ValueError):
        quant.resolve_mode("nvfp4", "cpu")


def test_summarize_counts_quantized_bytes():  # reference tests/test_quant.py:71-80
    layers = torch.nn.ModuleList(
        [
            quant.QuantLinear(64, 32, mode="int8", dtype=torch.float32, device="cpu"),
            torch.nn.Linear(64, 8, bias=False),
        ]
    )
    report = quant.summarize(layers.modules())
    assert report["kernels"] == {"unused": 1}
    assert report["quantized_gib"] == round(64 * 32 / 1024**3, 3)


def test_make_linear_policy():
    assert isinstance(quant.make_linear(64, 32, quant="fp8", dtype=torch.bfloat16, device="cpu"), quant.QuantLinear)
    dense = quant.make_linear(64, 40, quant="fp8", dtype=torch.bfloat16, device="cpu")
    assert isinstance(dense, torch.nn.Linear) and not isinstance(dense, quant.QuantLinear)


def test_block_offset_table_cache_is_bounded():
    pb._LENGTHS.clear()
    for i in range(40):
        pb.block_offsets([i, i + 1], torch.device("cpu"))
    assert len(pb._LENGTHS) == pb._LENGTHS_MAX
    t = pb.block_offsets([3, 4], torch.device("cpu"))
    assert t.dtype == torch.int32 and t.tolist() == [3, 4]
