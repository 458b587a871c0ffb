"""The gated delta rule oracle against the reference's own CPU paths (CPU).

tests/golden/gdn.npz holds what d3trt.model.ops.recurrent_gated_delta_rule and
ops.chunk_gated_delta_rule (ops.py:287-360; transformers' torch fallbacks on the CPU)
returned on seeded inputs, with q/k repeated to HV heads as D3Core does. The fp64
restatement in oracle/gated_delta.py must agree with both to fp32 rounding.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden
from oracle.gated_delta import gated_delta_rule


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)


def golden_case(name: str):
    d = load_golden("gdn.npz")
    B, T, H, HV, K, V = (int(x) for x in d[f"{name}_meta"])
    q, k, v, beta = (bf16_bits_to_f32(d[f"{name}_{x}"]) for x in ("q", "k", "v", "beta"))
    h0 = d.get(f"{name}_h0")
    return dict(q=q, k=k, v=v, g=d[f"{name}_g"], beta=beta, h0=None if h0 is None else h0[None],
                dims=(B, T, H, HV, K, V), out=d)


@pytest.mark.parametrize("name", ["k64", "k128", "zero_init"])
def test_oracle_matches_reference_paths(name):
    c = golden_case(name)
    o, s = gated_delta_rule(c["q"], c["k"], c["v"], c["g"], c["beta"], c["h0"])
    for path in ("rec", "chunk"):
        assert np.abs(o - c["out"][f"{name}_o_{path}"]).max() <= 1e-6
        assert np.abs(s - c["out"][f"{name}_s_{path}"]).max() <= 1e-5


def test_oracle_identities():
    """beta = 0 leaves the state decaying only; zero input keeps a zero state."""
    rng = np.random.default_rng(0)
    B, T, H, K, V = 1, 6, 1, 64, 64
    q, k = rng.standard_normal((B, T, H, K)), rng.standard_normal((B, T, H, K))
    v = rng.standard_normal((B, T, H, V))
    g = -np.abs(rng.standard_normal((B, T, H)))
    h0 = rng.standard_normal((1, H, K, V))
    o, s = gated_delta_rule(q, k, v, g, np.zeros((B, T, H)), h0)
    assert np.allclose(s, h0 * np.exp(g.sum(1))[:, :, None, None])
    o, s = gated_delta_rule(q, k, v, g, np.ones((B, T, H)), None)
    assert np.isfinite(o).all()
    o0, s0 = gated_delta_rule(q, k, np.zeros_like(v), g, np.ones((B, T, H)), None)
    assert not o0.any() and not s0.any()
