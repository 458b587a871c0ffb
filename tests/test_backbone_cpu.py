"""CPU checks of the torch formulas d3_turbo_trt_b200.model.backbone keeps from
the model (no GPU): rotary tables and rotation, zero-centred RMSNorm, gated
RMSNorm and the causal depthwise convolution, each against transformers'
Qwen3.5 module on the same bf16 inputs, bit for bit."""

from __future__ import annotations

import pytest
import torch

from d3_turbo_trt_b200.model import backbone as bb

m = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")


def _cfg():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig

    return Qwen3_5TextConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                             rope_parameters={"rope_type": "default", "rope_theta": 10_000_000.0,
                                              "partial_rotary_factor": 0.25, "mrope_section": [11, 11, 10],
                                              "mrope_interleaved": True})


def test_rotary_matches_the_model():
    g = torch.Generator().manual_seed(0)
    rot = m.Qwen3_5TextRotaryEmbedding(_cfg())
    x = torch.randn(3, 40, 1024, generator=g).to(torch.bfloat16)
    pos = (700 + torch.arange(40))[None].expand(3, -1)
    # the module forms its tables with an fp32 matmul, whose CPU precision is a global torch
    # setting other code may lower: pin it for the reference, and allow one bf16 ulp
    saved = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    try:
        cos_ref, sin_ref = rot(x, pos[None].expand(3, -1, -1))
    finally:
        torch.set_float32_matmul_precision(saved)
    cos, sin = bb.rotary_tables(bb.BackboneConfig(), pos, torch.bfloat16)
    for got, want in ((cos, cos_ref), (sin, sin_ref)):
        d = (got.view(torch.int16).int() - want.view(torch.int16).int()).abs()
        assert int(d.max()) <= 1 and float((d == 0).float().mean()) > 0.99
    q = torch.randn(3, 8, 40, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(3, 2, 40, 128, generator=g).to(torch.bfloat16)
    qr, kr = m.apply_rotary_pos_emb(q, k, cos_ref, sin_ref)
    qo, ko = bb.apply_rotary(q, k, cos_ref, sin_ref)
    assert torch.equal(qo, qr) and torch.equal(ko, kr)


def test_norms_match_the_model():
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(64, 1024, generator=g) * 3).to(torch.bfloat16)
    n = m.Qwen3_5RMSNorm(1024).to(torch.bfloat16)
    n.weight.data = (torch.randn(1024, generator=g) * 0.1).to(torch.bfloat16)
    assert torch.equal(bb.rms_norm(x, n.weight.data, 1e-6), n(x))
    z = torch.randn(64, 128, generator=g).to(torch.bfloat16)
    c = torch.randn(64, 128, generator=g).to(torch.bfloat16)
    gn = m.Qwen3_5RMSNormGated(128).to(torch.bfloat16)
    gn.weight.data = (1 + torch.randn(128, generator=g) * 0.1).to(torch.bfloat16)
    assert torch.equal(bb.gated_rms_norm(c, z, gn.weight.data, 1e-6), gn(c, z))


def test_causal_conv_matches_the_reference_formula():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(3, 96, 30, generator=g).to(torch.bfloat16)
    w = (torch.randn(96, 4, generator=g) * 0.5).to(torch.bfloat16)
    ref = torch.nn.functional.silu(torch.nn.functional.conv1d(x, w.unsqueeze(1), None, padding=3, groups=96)[..., :30])
    assert torch.equal(bb.causal_conv1d(x, w), ref)
