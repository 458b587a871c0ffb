"""Producer-side oracle (numpy) for the fused norm/gate -> activation-quant kernels — test infrastructure only.

Every QuantLinear input of the model is produced by one of two element-wise
ops, restated here from the reference's own bf16-exact formulation of the
eager forward (reference/d3_kernels.py; HF Qwen3_5RMSNorm,
transformers/models/qwen3_5/modeling_qwen3_5.py:711-725):

* add_rmsnorm  (reference/d3_kernels.py:97-142, :145-170): hidden =
  bf16(residual + delta); rstd = rsqrt(mean(hidden^2) + eps);
  normed = bf16((hidden * rstd) * (1 + w)), all in fp32, optional row mask
  multiplying the normed rows of padding by 0. The mean is taken over an fp64 sum
  of squares (each bf16 square exact in fp64) rounded once to fp32 — the reference itself fixes no
  summation order (it reproduces one GPU library's order); rsqrt is correctly
  rounded (fp64 then one rounding), as the reference's ``rsqrt_rn`` (:36-39).
* sigmoid_gate (reference/d3_kernels.py:467-525, core.py:297):
  y = bf16(attn * bf16(1 / (1 + exp(-gate)))), fp32 arithmetic.

The fused kernels then quantise those bf16 rows exactly as ``quantize_rows``
(oracle/quant.py) does.
"""

from __future__ import annotations

import numpy as np

from .quant import bf16_round, quantize_rows


def add_rmsnorm(residual: np.ndarray, delta: np.ndarray | None, weight_plus_one: np.ndarray, eps: float,
                rowmask: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """(hidden, normed) as float32 arrays holding bf16 values ([M, K] each)."""
    x = np.asarray(residual, dtype=np.float32)
    if delta is not None:
        x = bf16_round((x + np.asarray(delta, dtype=np.float32)).astype(np.float32))
    k = x.shape[1]
    sumsq = (x.astype(np.float64) ** 2).sum(axis=1, keepdims=True)
    var = (sumsq / k).astype(np.float32)
    rstd = (1.0 / np.sqrt((var + np.float32(eps)).astype(np.float32).astype(np.float64))).astype(np.float32)
    w1 = np.asarray(weight_plus_one, dtype=np.float32).reshape(1, -1)
    normed = bf16_round(((x * rstd).astype(np.float32) * w1).astype(np.float32))
    if rowmask is not None:
        keep = (np.asarray(rowmask).reshape(-1, 1) != 0).astype(np.float32)
        normed = (normed * keep).astype(np.float32)  # as the reference: y * keep (negative y -> -0.0)
    return x, normed


def add_rmsnorm_quant(residual, delta, weight_plus_one, eps, mode, rowmask=None):
    """(hidden, q, scale): the normed rows quantised per row like quantize_rows."""
    hidden, normed = add_rmsnorm(residual, delta, weight_plus_one, eps, rowmask)
    q, s = quantize_rows(normed, mode)
    return hidden, q, s


def sigmoid_gate(attn: np.ndarray, gate: np.ndarray) -> np.ndarray:
    """[B, T, H, D] attention output and gate -> [B*T, H*D] gated rows (bf16 values in float32)."""
    a = np.asarray(attn, dtype=np.float32)
    g = np.asarray(gate, dtype=np.float32)
    with np.errstate(over="ignore"):
        s = bf16_round((np.float32(1.0) / (np.float32(1.0) + np.exp(-g))).astype(np.float32))
    y = bf16_round((a * s).astype(np.float32))
    b, t, h, d = y.shape
    return y.reshape(b * t, h * d)


def sigmoid_gate_quant(attn, gate, mode):
    """(q, scale) of the gated rows."""
    return quantize_rows(sigmoid_gate(attn, gate), mode)
