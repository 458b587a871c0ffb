"""GPU parity of the GDN causal convolution + SiLU kernel (d3b_causal_conv1d_silu)
against the reference's torch form (d3trt/model/ops.py:266-285: F.conv1d over the
channel-major [B, C, L] input, cut to L, then SiLU), for the state pass (no tail)
and the question pass (the snapshot's tail concatenated in front, shared by all
rows or one per row). The kernel sums in fp32 in kernel order, so its bf16 results
may differ from the library convolution's by one bf16 ulp where the fp32 sums
round differently; they must agree within that and be identical almost
everywhere."""

from __future__ import annotations

import pytest
import torch

from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.model.backbone import causal_conv1d
from d3_turbo_trt_b200.model.conv import causal_conv1d_silu

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ulps(a, b):
    return (a.view(torch.int16).int() - b.view(torch.int16).int()).abs()


def _check(got, want):
    d = _ulps(got, want)
    assert int(d.max()) <= 1 and float((d == 0).float().mean()) > 0.995


@pytest.mark.parametrize("B,T,C,W", [(1, 4096, 2048, 4), (1, 37, 520, 3), (3, 1, 64, 4), (2, 70, 1032, 5)])
def test_state_pass_against_torch(B, T, C, W):
    g = torch.Generator().manual_seed(B * 1000 + T)
    x = torch.randn(B, T, C, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(C, W, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    got = causal_conv1d_silu(x, w)
    want = causal_conv1d(x.transpose(1, 2), w).transpose(1, 2)
    _check(got, want)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("shared", [True, False])
def test_question_pass_with_tail(shared):
    g = torch.Generator().manual_seed(5)
    B, T, C, W = 17, 48, 1536, 4
    state = torch.randn(1 if shared else B, 200, C, generator=g).to(torch.bfloat16).to(DEV)
    x = torch.randn(B, T, C, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(C, W, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    tail = state[:, -(W - 1):, :].transpose(1, 2)  # [1 or B, C, W-1] strided view, as the backbone keeps it
    got = causal_conv1d_silu(x, w, tail)
    joined = torch.cat([tail.expand(B, -1, -1), x.transpose(1, 2)], dim=-1)
    want = causal_conv1d(joined, w)[:, :, W - 1:].transpose(1, 2)
    _check(got, want)
    # the input read through row and token strides (a slice of a wider buffer)
    wide = torch.randn(B, T, C + 64, generator=g).to(torch.bfloat16).to(DEV)
    got2 = causal_conv1d_silu(wide[..., :C], w, tail)
    joined2 = torch.cat([tail.expand(B, -1, -1), wide[..., :C].transpose(1, 2)], dim=-1)
    _check(got2, causal_conv1d(joined2, w)[:, :, W - 1:].transpose(1, 2))
    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,I", [(300, 2048), (77, 17408), (5, 512)])
def test_silu_mul_quant_against_torch(M, I):
    """SiLU(gate) * up (the MLP, bf16 as torch computes it) and its per-row codes."""
    from d3_turbo_trt_b200.model import fused, quant

    g = torch.Generator().manual_seed(M)
    gu = (torch.randn(M, 2 * I, generator=g) * 3).to(torch.bfloat16).to(DEV)
    want = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    act = fused.silu_mul(gu)
    _check(act, want)
    for mode in ("fp8", "int8"):
        q, s = fused.silu_mul_quant(gu, mode)
        rq, rs = quant.quantize_rows(act, mode)  # the codes of the kernel's own rows, bit for bit
        assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8)) and torch.equal(s, rs)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,H,D", [(300, 16, 128), (41, 48, 128), (9, 8, 64), (7, 4, 256)])
def test_gated_rmsnorm_quant_against_torch(M, H, D):
    """Qwen3_5RMSNormGated per head on token rows, and the rows' codes for out_proj."""
    from d3_turbo_trt_b200.model import fused, quant
    from d3_turbo_trt_b200.model.backbone import gated_rms_norm

    g = torch.Generator().manual_seed(M + H)
    x = (torch.randn(M, H * D, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    z = torch.randn(M, H * D, generator=g).to(torch.bfloat16).to(DEV)
    w = (1 + torch.randn(D, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    want = gated_rms_norm(x.reshape(-1, D), z.reshape(-1, D), w, 1e-6).reshape(M, H * D)
    out = fused.gated_rmsnorm(x, z, w, 1e-6, D)
    _check(out, want)
    for mode in ("fp8", "int8"):
        q, s = fused.gated_rmsnorm_quant(x, z, w, 1e-6, D, mode)
        rq, rs = quant.quantize_rows(out, mode)
        assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8)) and torch.equal(s, rs)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("rows,T,heads,stride_heads", [(1, 300, 32, 2), (37, 48, 4, 1), (5, 7, 8, 2), (3, 9, 3, 1),
                                                      (2, 5, 19, 2)])
def test_qk_norm_rope_against_torch(rows, T, heads, stride_heads):
    """q_norm / k_norm (Qwen3_5RMSNorm per head) then the partial rotary embedding (rd = 32 of
    128) in one kernel, against the backbone's torch restatement of the model's functions.
    The two sum each head's squares in different orders, so a normalised value can land one
    bf16 step away; the rotary sum of two such terms then moves by up to about two steps at
    the terms' magnitude (the head's), not the result's. So: every value within 2^-5 of its
    head's largest value, and under 2 % of the values differing at all. The input is a
    strided slice (the query half of q_proj's output) when stride_heads is 2."""
    from d3_turbo_trt_b200.model import fused
    from d3_turbo_trt_b200.model.backbone import BackboneConfig, apply_rotary, rms_norm, rotary_tables

    D = 128
    g = torch.Generator().manual_seed(rows * 7 + T)
    full = (torch.randn(rows, T, heads, stride_heads * D, generator=g) * 2.0).to(torch.bfloat16).to(DEV)
    x = full[..., :D]
    w = (torch.randn(D, generator=g) * 0.2).to(torch.bfloat16).to(DEV)
    positions = (torch.arange(T)[None] + 4096 * torch.arange(rows)[:, None]).to(DEV)
    cos, sin = rotary_tables(BackboneConfig(), positions, torch.bfloat16)
    assert cos.shape[-1] == 32
    want, _ = apply_rotary(rms_norm(x, w, 1e-6).transpose(1, 2), x.transpose(1, 2)[:, :1], cos, sin)
    got = fused.qk_norm_rope(x, w, cos, sin, 1e-6)
    assert got.shape == (rows, T, heads, D) and got.is_contiguous()
    got_h, want_f = got.transpose(1, 2).float(), want.float()
    diff = (got_h - want_f).abs()
    head_max = want_f.abs().amax(-1, keepdim=True)
    assert bool((diff <= head_max * 2.0 ** -5).all()), float((diff / head_max).max())
    assert float((diff > 0).float().mean()) < 0.02
    assert _lib.device_error() == 0


def test_silu_mul_every_bf16_gate():
    """Every finite bf16 value as the gate (up = 1): the kernel's SiLU equals
    bf16(g / (1 + exp(-g))) in fp32 with torch's exp and IEEE division bit for bit, values
    next to bf16 rounding boundaries, large |g|, zeros and subnormals included."""
    from d3_turbo_trt_b200.model import fused

    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
    g = bits.view(torch.bfloat16)
    g = g[torch.isfinite(g.float())]
    n = g.numel()
    I = 8 * ((n + 7) // 8)
    gate = torch.zeros(I, dtype=torch.bfloat16)
    gate[:n] = g
    per = 4096  # rows of 4096 gates each (the kernel's rows hold up to 24576)
    nrow = I // per + (1 if I % per else 0)
    gates = torch.zeros(nrow * per, dtype=torch.bfloat16)
    gates[:I] = gate
    gates = gates.reshape(nrow, per)
    gu = torch.cat([gates, torch.ones_like(gates)], 1).to(DEV)
    act = fused.silu_mul(gu)
    gf = gates.to(DEV).float()
    want = (gf / (1.0 + torch.exp(-gf))).to(torch.bfloat16)
    assert torch.equal(act.view(torch.int16), want.view(torch.int16)), int((act != want).sum())
    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,HV,stride", [(12240, 48, 16480), (37, 16, 16), (5, 48, 64)])
def test_gdn_gates_against_torch(M, HV, stride):
    """beta = b.sigmoid() and g = -A_log.float().exp() * softplus(a.float() + dt_bias) of the GDN
    layer (d3trt/model/core.py:341-342) in one kernel, a and b read as row slices of a wider
    projection: both bit-identical to torch's element-wise ops, softplus's linear branch
    (x > 20) and large negative gates included."""
    from d3_turbo_trt_b200.model import fused

    g = torch.Generator().manual_seed(M + HV)
    proj = (torch.randn(M, stride + 2 * HV, generator=g) * 6).to(torch.bfloat16)
    proj[0, :HV] = 25.0  # softplus's x > 20 branch
    proj[1, :HV] = -90.0
    proj = proj.to(DEV)
    a, b = proj[:, :HV], proj[:, stride - HV:stride] if stride >= 2 * HV else proj[:, HV:2 * HV]
    A_log = torch.log(torch.rand(HV, generator=g) * 1.95 + 0.05).to(torch.bfloat16).to(DEV)
    dt_bias = (1 + torch.randn(HV, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    want_beta = b.sigmoid()
    want_g = -A_log.float().exp() * torch.nn.functional.softplus(a.float() + dt_bias)
    got_g, got_beta = fused.gdn_gates(a, b, -A_log.float().exp(), dt_bias.float())
    assert torch.equal(got_beta.view(torch.int16), want_beta.contiguous().view(torch.int16))
    assert torch.equal(got_g, want_g)
    assert _lib.device_error() == 0
