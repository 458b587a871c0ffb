"""W8A8 quantisation oracle (numpy) — test infrastructure only.

Restates d3trt/model/quant.py:
* quantize_rows    (quant.py:92-100)
* quantize_weight  (quant.py:77-89)
* QuantLinear._emulated (quant.py:158-162): y = (acc * s_a) * s_w, fp32
* torch._int_mm semantics (quant.py:196): exact int32 accumulators
and the float32 -> float8_e4m3fn conversion that ``.to(torch.float8_e4m3fn)``
performs (round to nearest even; e4m3fn: bias 7, no infinities, max 448,
subnormal step 2^-9, NaN = 0x7F/0xFF), written from the OCP FP8 format
definition.
"""

from __future__ import annotations

import numpy as np

FP8_MAX = np.float32(448.0)
INT8_MAX = np.float32(127.0)
EPS = np.float32(1e-12)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn bit patterns (uint8), RNE; |x| > 448 saturates to 448."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    sign = (np.signbit(x)).astype(np.uint8) << 7
    nan = np.isnan(x)
    a = np.where(nan, 0.0, a)
    # exponent of the quantisation step: normals use 3 mantissa bits, the
    # subnormal range (|x| < 2^-6) a fixed step of 2^-9
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)
    step = np.exp2(e - 3.0)
    m = np.rint(a / step)  # half to even
    v = np.minimum(m * step, 448.0)
    # bit pattern of the rounded value
    with np.errstate(divide="ignore"):
        ev = np.floor(np.log2(np.where(v > 0, v, 1.0)))
    normal = v >= 2.0**-6
    exp_field = np.where(normal, ev + 7.0, 0.0)
    mant = np.where(normal, v / np.exp2(ev) * 8.0 - 8.0, v / 2.0**-9)
    bits = (exp_field.astype(np.int64) << 3) | np.rint(mant).astype(np.int64)
    bits = np.where(v == 0, 0, bits).astype(np.uint8) | sign
    return np.where(nan, np.uint8(0x7F) | sign, bits).astype(np.uint8)


def e4m3_decode(bits: np.ndarray) -> np.ndarray:
    """e4m3fn bit patterns -> float32 values."""
    b = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    exp_field = (b >> 3) & 0xF
    mant = b & 0x7
    val = np.where(exp_field == 0, mant * 2.0**-9, (1.0 + mant / 8.0) * np.exp2(exp_field - 7.0))
    val = np.where((exp_field == 0xF) & (mant == 0x7), np.nan, val)
    return (sign * val).astype(np.float32)


def quantize_rows(x: np.ndarray, mode: str) -> tuple[np.ndarray, np.ndarray]:
    """[M, K] -> (q [M, K] uint8 e4m3 bits or int8, scale [M, 1] float32) (quant.py:92-100)."""
    xf = np.asarray(x, dtype=np.float32)
    amax = np.maximum(np.abs(xf).max(axis=1, keepdims=True), EPS).astype(np.float32)
    if mode == "fp8":
        scale = (amax / FP8_MAX).astype(np.float32)
        v = np.clip((xf / scale).astype(np.float32), -FP8_MAX, FP8_MAX)
        return e4m3_encode(v), scale
    scale = (amax / INT8_MAX).astype(np.float32)
    v = np.clip(np.rint((xf / scale).astype(np.float32)), -INT8_MAX, INT8_MAX)
    return v.astype(np.int8), scale


def quantize_weight(w: np.ndarray, mode: str) -> tuple[np.ndarray, np.ndarray]:
    """[N, K] -> (q [N, K], scale [N]) (quant.py:77-89)."""
    if mode not in ("fp8", "int8"):
        raise ValueError(f"cannot quantize weights to {mode!r}")
    q, s = quantize_rows(w, mode)
    return q, s[:, 0]


def dequant_codes(q: np.ndarray, mode: str) -> np.ndarray:
    return e4m3_decode(q) if mode == "fp8" else np.asarray(q, dtype=np.float32)


def int_gemm(qa: np.ndarray, qw: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators of int8 [M,K] x int8 [N,K]^T (torch._int_mm, quant.py:196)."""
    acc = np.asarray(qa, dtype=np.int64) @ np.asarray(qw, dtype=np.int64).T
    return acc.astype(np.int32)


def w8a8_linear(
    qa: np.ndarray, sa: np.ndarray, qw: np.ndarray, sw: np.ndarray, mode: str
) -> np.ndarray:
    """fp32 result before the final cast: (acc * s_a) * s_w (quant.py:158-162, :196-197).

    The accumulator is exact (int64 for int8, float64 for e4m3 products, then
    rounded once to float32), so it equals the reference's fp32 accumulation
    whenever that is exact and differs only by fp32 summation rounding else.
    """
    if mode == "int8":
        acc = int_gemm(qa, qw).astype(np.float32)
    else:
        acc = (dequant_codes(qa, mode).astype(np.float64) @ dequant_codes(qw, mode).astype(np.float64).T).astype(
            np.float32
        )
    sa = np.asarray(sa, dtype=np.float32).reshape(-1, 1)
    sw = np.asarray(sw, dtype=np.float32).reshape(1, -1)
    return ((acc * sa).astype(np.float32) * sw).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32 values."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return rounded.astype(np.uint32).view(np.float32)
