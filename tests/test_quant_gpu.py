"""GPU parity of the W8A8 path: activation quant bit-exact with quantize_rows
(d3trt/model/quant.py:92-100), int32 accumulators bit-exact with torch._int_mm,
e4m3 GEMM within 2e-2 max-abs of the fp32 reference before rounding, and the
bf16 outputs within one bf16 ulp of the rounded reference."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import quant as oq

from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.model import quant

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _codes(q: torch.Tensor) -> np.ndarray:
    return q.view(torch.uint8).cpu().numpy() if q.dtype == torch.float8_e4m3fn else q.cpu().numpy().view(np.uint8)


def _cfg2_activations(rows=4096, k=5120, seed=0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    cols = torch.randperm(k, generator=g)[: k // 100]
    x[:, cols] *= 20.0
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_act_quant_golden_bit_exact(mode):
    g = load_golden("quant.npz")
    x = bf16_from_bits(g["rows_x_bf16"]).to(DEV)
    q, s = quant.quantize_rows(x, mode)
    assert np.array_equal(s.cpu().numpy(), g[f"rows_s_{mode}"])
    assert np.array_equal(_codes(q), g[f"rows_q_{mode}"].view(np.uint8))
    q32, s32 = quant.quantize_rows(torch.from_numpy(g["rows_x_f32"]).to(DEV), mode)
    assert np.array_equal(s32.cpu().numpy(), g[f"rows32_s_{mode}"])
    assert np.array_equal(_codes(q32), g[f"rows32_q_{mode}"].view(np.uint8))


@pytest.mark.parametrize("mode", ["fp8", "int8"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_act_quant_cfg2_bit_exact(mode, dtype):
    x = _cfg2_activations().to(dtype)
    q, s = quant.quantize_rows(x.to(DEV), mode)
    rq, rs = oq.quantize_rows(x.float().numpy(), mode)
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(_codes(q), rq.view(np.uint8))


@pytest.mark.parametrize("k", [8, 4096, 5120, 5128, 6144, 6152, 17408])
def test_act_quant_bf16_row_lengths_bit_exact(k):
    """bf16 rows up to 6144 wide go through the one-pass register kernel (three
    sizes of it), longer rows through the two-pass kernel; a padded row pitch
    exercises both with ldx > K."""
    x = _cfg2_activations(rows=67, k=k, seed=k)
    padded = torch.zeros(67, k + 64, dtype=torch.bfloat16)
    padded[:, :k] = x
    for src in (x.to(DEV), padded.to(DEV)[:, :k]):
        for mode in ("fp8", "int8"):
            q, s = quant.quantize_rows(src, mode)
            rq, rs = oq.quantize_rows(x.float().numpy(), mode)
            assert np.array_equal(s.cpu().numpy(), rs)
            assert np.array_equal(_codes(q), rq.view(np.uint8))


def test_act_quant_strided_rows_and_zero_row():
    base = torch.randn(33, 200, dtype=torch.bfloat16)
    base[7] = 0
    x = base.to(DEV)[:, :136]  # row pitch 200, K = 136 (tail past the vector loop)
    for mode in ("fp8", "int8"):
        q, s = quant.quantize_rows(x, mode)
        rq, rs = oq.quantize_rows(base[:, :136].float().numpy(), mode)
        assert np.array_equal(s.cpu().numpy(), rs)
        assert np.array_equal(_codes(q), rq.view(np.uint8))
        assert np.all(_codes(q)[7] == 0)
        assert s[7].item() == pytest.approx(1e-12 / (448.0 if mode == "fp8" else 127.0))


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_weight_quant_golden(mode):
    g = load_golden("quant.npz")
    w = bf16_from_bits(g["w_bf16"]).to(DEV)
    q, s = quant.quantize_weight(w, mode)
    assert s.shape == (96,)
    assert np.array_equal(s.cpu().numpy(), g[f"w_s_{mode}"])
    assert np.array_equal(_codes(q), g[f"w_q_{mode}"].view(np.uint8))


def _rand_codes(rows, k, mode, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    return oq.quantize_rows(x.numpy(), mode)


def _to_dev_codes(q: np.ndarray, mode: str) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(q).view(np.uint8 if mode == "fp8" else np.int8))
    return (t.view(torch.float8_e4m3fn) if mode == "fp8" else t).to(DEV)


@pytest.mark.parametrize("shape", [(300, 272, 320), (1, 16, 16), (129, 512, 4096), (256, 256, 128)])
def test_int8_accumulators_bit_exact(shape):
    m, n, k = shape
    qa, _ = _rand_codes(m, k, "int8", 1)
    qw, _ = _rand_codes(n, k, "int8", 2)
    acc = quant.scaled_mm(_to_dev_codes(qa, "int8"), _to_dev_codes(qw, "int8"), None, None, out_dtype=torch.int32)
    assert np.array_equal(acc.cpu().numpy(), oq.int_gemm(qa, qw))


@pytest.mark.parametrize("shape", [(512, 256, 128), (600, 272, 320), (777, 1040, 4096), (1030, 528, 17408)])
def test_int8_pair_tiles_bit_exact(shape):
    """M >= 512 runs on CTA pairs (256 x 256 tiles): ragged M leaves the second CTA's
    rows past the end, ragged N the second half of B."""
    m, n, k = shape
    qa, _ = _rand_codes(m, k, "int8", 11)
    qw, _ = _rand_codes(n, k, "int8", 12)
    a, w = _to_dev_codes(qa, "int8"), _to_dev_codes(qw, "int8")
    acc = quant.scaled_mm(a, w, None, None, out_dtype=torch.int32)
    if m * n * k <= 600 * 272 * 320:
        assert np.array_equal(acc.cpu().numpy(), oq.int_gemm(qa, qw))
    assert torch.equal(acc, torch._int_mm(a, w.t()))
    assert _lib.device_error() == 0


@pytest.mark.parametrize("mode", ["fp8", "int8"])
@pytest.mark.parametrize("shape", [(300, 272, 320), (77, 13824 // 8, 5120), (600, 272, 320), (1030, 528, 1024)])
def test_w8a8_fp32_and_bf16_outputs(mode, shape):
    m, n, k = shape
    qa, sa = _rand_codes(m, k, mode, 3)
    qw, sw = _rand_codes(n, k, mode, 4)
    ref = oq.w8a8_linear(qa, sa, qw, sw, mode)
    a, w = _to_dev_codes(qa, mode), _to_dev_codes(qw, mode)
    sa_t, sw_t = torch.from_numpy(sa).to(DEV), torch.from_numpy(sw).to(DEV)
    y32 = quant.scaled_mm(a, w, sa_t, sw_t, out_dtype=torch.float32).cpu().numpy()
    if mode == "int8":
        assert np.array_equal(y32, ref)
    else:
        assert np.abs(y32 - ref).max() <= 2e-2
        assert np.abs(y32 - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
    y16 = quant.scaled_mm(a, w, sa_t, sw_t, out_dtype=torch.bfloat16).float().cpu().numpy()
    ref16 = oq.bf16_round(ref)
    if mode == "int8":
        assert np.array_equal(y16, ref16)
    else:
        # the bf16 store is the kernel's own fp32 result rounded once; against the
        # reference: the fp32 tolerance above plus the two roundings (<= 2 ulp)
        assert np.array_equal(y16, oq.bf16_round(y32))
        ulp = np.abs(oq.bf16_round(ref * (1 + 2.0**-7)) - ref16) + 1e-30
        assert np.all(np.abs(y16 - ref16) <= 2 * ulp + 1e-5 * max(1.0, np.abs(ref).max()))


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_quant_linear_golden(mode):
    g = load_golden("quant.npz")
    w = bf16_from_bits(g["w_bf16"]).to(DEV)
    x = bf16_from_bits(g["lin_x_bf16"]).to(DEV)
    layer = quant.QuantLinear(256, 96, mode=mode, dtype=torch.bfloat16, device=DEV)
    layer.load_full(w)
    y = layer(x)
    assert y.shape == (3, 5, 96) and y.dtype == torch.bfloat16
    assert layer.kernel == "sm100a"
    ref = bf16_from_bits(g[f"lin_y_{mode}_bf16"]).float().numpy().reshape(3, 5, 96)
    got = y.float().cpu().numpy()
    if mode == "int8":
        assert np.array_equal(got, ref)
    else:
        assert np.abs(got - ref).max() <= 2e-2


@pytest.mark.parametrize("mode,limit", [("fp8", 0.06), ("int8", 0.02)])
def test_quant_linear_matches_dense(mode, limit):  # reference tests/test_quant.py:15-26 on the GPU
    torch.manual_seed(0)
    weight = torch.randn(96, 256) * 0.02
    x = torch.randn(3, 5, 256, dtype=torch.bfloat16)
    layer = quant.QuantLinear(256, 96, mode=mode, dtype=torch.bfloat16, device=DEV)
    layer.load_full(weight.to(torch.bfloat16).to(DEV))
    out = layer(x.to(DEV)).float().cpu()
    ref = x.float() @ weight.t()
    assert float((out - ref).norm() / ref.norm()) < limit


def test_outlier_rows_and_zero_rows():  # reference tests/test_quant.py:29-40 on the GPU
    torch.manual_seed(0)
    weight = torch.randn(32, 64)
    x = torch.randn(4, 64)
    x[1] *= 1000.0
    x[3] = 0.0
    layer = quant.QuantLinear(64, 32, mode="int8", dtype=torch.float32, device=DEV)
    layer.load_full(weight.to(DEV))
    out = layer(x.to(DEV)).cpu()
    ref = x @ weight.t()
    assert float((out[0] - ref[0]).norm() / ref[0].norm()) < 0.02
    assert torch.all(out[3] == 0)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_cfg2_full_size(mode):
    """[4096, 5120] x [13824, 5120]^T, 1% outlier channels."""
    x = _cfg2_activations()
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(13824, 5120, generator=g) * 0.02).to(torch.bfloat16)
    layer = quant.QuantLinear(5120, 13824, mode=mode, dtype=torch.bfloat16, device=DEV)
    layer.load_full(w.to(DEV))
    qa, sa = quant.quantize_rows(x.to(DEV), mode)
    rows = torch.tensor([0, 1, 127, 128, 2047, 4095])
    qa_np = _codes(qa)[rows.numpy()]
    qw_np = _codes(layer.weight)
    if mode == "int8":
        qa_np, qw_np = qa_np.view(np.int8), qw_np.view(np.int8)
        acc = quant.scaled_mm(qa, layer.weight, None, None, out_dtype=torch.int32)
        assert np.array_equal(acc[rows.to(DEV)].cpu().numpy(), oq.int_gemm(qa_np, qw_np))
        # the whole [4096, 13824] int32 accumulator, bit for bit, against torch._int_mm
        # (exact integer arithmetic, the reference's own INT8 call: quant.py:190-197)
        assert torch.equal(acc, torch._int_mm(qa, layer.weight.t()))
    y32 = quant.scaled_mm(qa, layer.weight, sa, layer.weight_scale, out_dtype=torch.float32)
    ref = oq.w8a8_linear(qa_np, sa[rows.to(DEV)].cpu().numpy(), qw_np, layer.weight_scale.cpu().numpy(), mode)
    got = y32[rows.to(DEV)].cpu().numpy()
    if mode == "int8":
        assert np.array_equal(got, ref)
    else:
        assert np.abs(got - ref).max() <= 2e-2
    y = layer(x.to(DEV))
    assert torch.equal(y, y32.to(torch.bfloat16))
    # the kernel against torch._scaled_mm (the reference's GPU call), fp8 only
    if mode == "fp8":
        ts = torch._scaled_mm(qa, layer.weight.t(), scale_a=sa, scale_b=layer.weight_scale[None, :],
                              out_dtype=torch.bfloat16)
        # both round to bf16: allow one bf16 ulp of the larger magnitude
        assert float(((ts.float() - y.float()).abs() / y.float().abs().clamp_min(1.0)).max()) <= 2.0**-7
    assert _lib.device_error() == 0
