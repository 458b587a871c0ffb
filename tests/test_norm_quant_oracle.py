"""CPU checks of the fused-producer oracle (oracle/norm_quant.py): against an
independent torch formulation of the eager model ops (Qwen3_5RMSNorm after a
bf16 residual add, modeling_qwen3_5.py:711-725, and attn * sigmoid(gate)), and
against the fixture recorded from the modules themselves and the reference's
quantize_rows (tests/golden/norm_quant.npz)."""

from __future__ import annotations

import numpy as np
import torch

from conftest import load_golden
from oracle import norm_quant as onq
from oracle import quant as oq


def _ulp_diff_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    ia = np.asarray(a, np.float32).view(np.int32) >> 16
    ib = np.asarray(b, np.float32).view(np.int32) >> 16
    return np.abs(ia.astype(np.int64) - ib.astype(np.int64))


def test_add_rmsnorm_oracle_matches_eager_formula():
    g = torch.Generator().manual_seed(0)
    M, K, eps = 64, 1024, 1e-6
    res = torch.randn(M, K, generator=g).to(torch.bfloat16)
    delta = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16)
    w = torch.randn(K, generator=g) * 0.1
    hidden, normed = onq.add_rmsnorm(res.float().numpy(), delta.float().numpy(), (1 + w).numpy(), eps)
    h = res + delta  # bf16 add (fp32 sum, one rounding)
    x = h.float()
    want = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w)).to(torch.bfloat16)
    assert np.array_equal(hidden, h.float().numpy())
    d = _ulp_diff_bf16(normed, want.float().numpy())
    assert d.max() <= 1 and (d == 0).mean() > 0.99  # the eager mean is an fp32 sum in another order


def test_add_rmsnorm_rowmask_and_quant_compose():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(8, 256, generator=g).to(torch.bfloat16).float().numpy()
    w1 = np.ones(256, np.float32)
    mask = np.array([1, 0, 1, 1, 0, 1, 1, 1])
    _, normed = onq.add_rmsnorm(x, None, w1, 1e-6, mask)
    assert np.all(normed[mask == 0] == 0)
    for mode in ("fp8", "int8"):
        h, q, s = onq.add_rmsnorm_quant(x, None, w1, 1e-6, mode, mask)
        rq, rs = oq.quantize_rows(normed, mode)
        assert np.array_equal(q, rq) and np.array_equal(s, rs) and np.array_equal(h, x)


def test_sigmoid_gate_oracle_matches_eager_formula():
    g = torch.Generator().manual_seed(2)
    a = torch.randn(2, 5, 4, 64, generator=g).to(torch.bfloat16)
    gt = (torch.randn(2, 5, 4, 64, generator=g) * 3).to(torch.bfloat16)
    got = onq.sigmoid_gate(a.float().numpy(), gt.float().numpy())
    want = (a * torch.sigmoid(gt)).reshape(10, 256).float().numpy()
    d = _ulp_diff_bf16(got, want)
    assert d.max() <= 1 and (d == 0).mean() > 0.99  # exp implementations may differ in the last fp32 bit


def _bf16(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits).astype(np.uint32) << 16).view(np.float32)


def test_oracle_pinned_to_model_modules():
    """tests/golden/norm_quant.npz was recorded from transformers' Qwen3_5RMSNorm
    after a bf16 residual add, the eager ``out * sigmoid(gate)`` and the
    reference's own quantize_rows (tests/golden/make_norm_golden.py)."""
    g = load_golden("norm_quant.npz")
    res, delta = _bf16(g["residual"]), _bf16(g["delta"])
    hidden, normed = onq.add_rmsnorm(res, delta, 1.0 + g["weight"], float(g["eps"]))
    assert np.array_equal(hidden, _bf16(g["hidden"]))
    d = _ulp_diff_bf16(normed, _bf16(g["normed"]))
    # the module's mean is an fp32 sum in its own order; the oracle's is exact
    assert d.max() <= 1 and (d == 0).mean() > 0.99
    gated = onq.sigmoid_gate(_bf16(g["attn"]), _bf16(g["gate"]))
    d = _ulp_diff_bf16(gated, _bf16(g["gated"]))
    assert d.max() <= 1 and (d == 0).mean() > 0.99
    # codes: identical wherever the rows themselves are identical
    for mode in ("fp8", "int8"):
        for name, rows in (("normed", normed), ("gated", gated)):
            q, s = onq.quantize_rows(rows, mode)
            same = np.all(rows == _bf16(g[name]), axis=1)
            assert same.mean() > 0.5
            assert np.array_equal(s[same], g[f"{name}_s_{mode}"][same])
            assert np.array_equal(q.view(np.uint8)[same], g[f"{name}_q_{mode}"].view(np.uint8)[same])
