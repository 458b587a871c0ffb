"""GPU parity of the fused producers (csrc/norm_quant.cu) through their C-ABI
entry points: residual add + Qwen3.5 RMSNorm (+ per-row quant) and
attn * sigmoid(gate) (+ per-row quant), against the numpy oracle
(oracle/norm_quant.py) bit-exactly, and against eager torch on the GPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import norm_quant as onq
from oracle import quant as oq

from d3_turbo_trt_b200.model import fused, quant

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _codes(q: torch.Tensor) -> np.ndarray:
    return q.view(torch.uint8).cpu().numpy() if q.dtype == torch.float8_e4m3fn else q.cpu().numpy().view(np.uint8)


def _inputs(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    res = (torch.randn(M, K, generator=g) * 2).to(torch.bfloat16)
    delta = torch.randn(M, K, generator=g).to(torch.bfloat16)
    cols = torch.randperm(K, generator=g)[: max(1, K // 100)]
    delta[:, cols] *= 20  # outlier channels, as the activations of BASELINE config 2
    w1 = 1 + torch.randn(K, generator=g) * 0.1
    return res, delta, w1


@pytest.mark.parametrize("K", [1024, 4096, 5120, 6144])
@pytest.mark.parametrize("with_delta", [True, False])
def test_add_rmsnorm_bit_exact_with_oracle(K, with_delta):
    res, delta, w1 = _inputs(131, K, K)
    d = delta if with_delta else None
    hidden, normed = fused.add_rmsnorm(res.to(DEV), d.to(DEV) if with_delta else None, w1, 1e-6)
    oh, on = onq.add_rmsnorm(res.float().numpy(), d.float().numpy() if with_delta else None, w1.numpy(), 1e-6)
    assert np.array_equal(hidden.float().cpu().numpy(), oh)
    assert np.array_equal(normed.float().cpu().numpy(), on)
    for mode in ("fp8", "int8"):
        h2, q, s = fused.add_rmsnorm_quant(res.to(DEV), d.to(DEV) if with_delta else None, w1, 1e-6, mode)
        rq, rs = oq.quantize_rows(on, mode)
        assert np.array_equal(s.cpu().numpy(), rs)
        assert np.array_equal(_codes(q), rq.view(np.uint8))
        assert torch.equal(h2.cpu(), hidden.cpu())


def test_add_rmsnorm_rowmask_and_eager_torch():
    res, delta, w1 = _inputs(64, 5120, 5)
    mask = torch.tensor([i % 3 != 0 for i in range(64)], dtype=torch.int32)
    hidden, normed = fused.add_rmsnorm(res.to(DEV), delta.to(DEV), w1, 1e-6, rowmask=mask.to(DEV))
    _, on = onq.add_rmsnorm(res.float().numpy(), delta.float().numpy(), w1.numpy(), 1e-6, mask.numpy())
    assert np.array_equal(normed.float().cpu().numpy(), on)
    # eager torch on the GPU (fp32 mean in its own order): within one bf16 ulp
    h = res.to(DEV) + delta.to(DEV)
    x = h.float()
    want = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w1.to(DEV)).to(torch.bfloat16)
    want = want * mask.to(DEV)[:, None].to(torch.bfloat16)
    ia = normed.view(torch.int16).int()
    ib = want.view(torch.int16).int()
    assert (ia - ib).abs().max().item() <= 1
    assert torch.equal(hidden, h)


def test_fused_quant_feeds_quant_linear():
    res, delta, w1 = _inputs(96, 5120, 9)
    g = torch.Generator().manual_seed(11)
    w = (torch.randn(1024, 5120, generator=g) * 0.02).to(torch.bfloat16)
    for mode in ("fp8", "int8"):
        layer = quant.QuantLinear(5120, 1024, mode=mode, dtype=torch.bfloat16, device=DEV)
        layer.load_full(w.to(DEV))
        _, normed = fused.add_rmsnorm(res.to(DEV), delta.to(DEV), w1, 1e-6)
        _, q, s = fused.add_rmsnorm_quant(res.to(DEV), delta.to(DEV), w1, 1e-6, mode)
        assert torch.equal(layer.forward_quantized(q, s), layer(normed))


def _gate_inputs(B, T, H, D, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16)  # attention output layout [B, H, T, D]
    qg = (torch.randn(B, T, H, 2 * D, generator=g) * 3).to(torch.bfloat16)  # q_proj output: query | gate per head
    return a, qg


@pytest.mark.parametrize("H,D", [(32, 128), (48, 128), (8, 64)])
def test_sigmoid_gate_matches_eager_and_oracle(H, D):
    B, T = 3, 37
    a, qg = _gate_inputs(B, T, H, D, H + D)
    attn = a.to(DEV).permute(0, 2, 1, 3)  # [B, T, H, D] view of the attention output
    gate = qg.to(DEV)[..., D:]  # [B, T, H, D] view into q_proj's output
    got = fused.sigmoid_gate(attn, gate)
    eager = (attn * torch.sigmoid(gate)).reshape(B, T, H * D)
    assert torch.equal(got, eager)  # same fp32 expf and IEEE division as the eager kernels
    orc = onq.sigmoid_gate(attn.float().cpu().numpy(), gate.float().cpu().numpy())
    d = (got.reshape(B * T, -1).view(torch.int16).int().cpu() - torch.from_numpy(orc).to(torch.bfloat16).view(torch.int16).int()).abs()
    assert d.max().item() <= 1
    for mode in ("fp8", "int8"):
        q, s = fused.sigmoid_gate_quant(attn, gate, mode)
        rq, rs = quant.quantize_rows(eager.reshape(B * T, H * D), mode)
        assert torch.equal(s, rs)
        assert np.array_equal(_codes(q), _codes(rq))


def test_unsupported_shapes_raise():
    x = torch.zeros(4, 6152, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError):
        fused.add_rmsnorm(x, None, torch.ones(6152), 1e-6)
    y = torch.zeros(4, 100, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError):
        fused.add_rmsnorm(y, None, torch.ones(100), 1e-6)
    with pytest.raises(RuntimeError):
        fused.add_rmsnorm(x.float(), None, torch.ones(6152), 1e-6)


def test_fused_producers_against_model_module_fixture():
    """The fused kernels on the inputs of tests/golden/norm_quant.npz (recorded
    from transformers' Qwen3_5RMSNorm, the eager gate and the reference's
    quantize_rows): rows within one bf16 ulp of the modules, codes and scales
    identical wherever the rows are identical."""
    from conftest import bf16_from_bits, load_golden

    g = load_golden("norm_quant.npz")
    res, delta = bf16_from_bits(g["residual"]).to(DEV), bf16_from_bits(g["delta"]).to(DEV)
    w1 = torch.from_numpy(1.0 + g["weight"])
    for mode in ("fp8", "int8"):
        hidden, q, s = fused.add_rmsnorm_quant(res, delta, w1, float(g["eps"]), mode)
        _, normed = fused.add_rmsnorm(res, delta, w1, float(g["eps"]))
        assert torch.equal(hidden.cpu(), bf16_from_bits(g["hidden"]))
        want = bf16_from_bits(g["normed"])
        ulps = (normed.cpu().view(torch.int16).int() - want.view(torch.int16).int()).abs()
        assert int(ulps.max()) <= 1
        same = (normed.cpu() == want).all(dim=1).numpy()
        assert same.mean() > 0.5
        assert np.array_equal(s.cpu().numpy().reshape(-1)[same], g[f"normed_s_{mode}"].reshape(-1)[same])
        assert np.array_equal(_codes(q)[same], g[f"normed_q_{mode}"].view(np.uint8)[same])
        attn, gate = bf16_from_bits(g["attn"]).to(DEV), bf16_from_bits(g["gate"]).to(DEV)
        qg, sg = fused.sigmoid_gate_quant(attn, gate, mode)
        gated = fused.sigmoid_gate(attn, gate).reshape(16, 256)
        want = bf16_from_bits(g["gated"])
        ulps = (gated.cpu().view(torch.int16).int() - want.view(torch.int16).int()).abs()
        assert int(ulps.max()) <= 1
        same = (gated.cpu() == want).all(dim=1).numpy()
        assert np.array_equal(sg.cpu().numpy().reshape(-1)[same], g[f"gated_s_{mode}"].reshape(-1)[same])
        assert np.array_equal(_codes(qg)[same], g[f"gated_q_{mode}"].view(np.uint8)[same])
