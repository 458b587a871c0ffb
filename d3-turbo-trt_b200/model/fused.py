"""Fused producers of the W8A8 linears' inputs (sm_100a kernels in csrc/norm_quant.cu).

Every ``QuantLinear`` input of the model comes out of one of two element-wise
ops; these functions compute them and, for the ``*_quant`` forms, the
per-row activation quantisation of the consuming linear in the same pass, so
the bf16 normed / gated rows never travel through HBM:

* ``add_rmsnorm(residual, delta, weight_plus_one, eps, rowmask=None)`` ->
  ``(hidden, normed)``: drop-in for reference/d3_kernels.py:145-170 (residual
  add + zero-centred RMSNorm of Qwen3.5).
* ``add_rmsnorm_quant(..., mode)`` -> ``(hidden, q, scale)``: the same, with
  ``normed`` quantised as ``quantize_rows`` (d3trt/model/quant.py:92-100) would;
  feed ``QuantLinear.forward_quantized(q, scale)`` of q/k/v_proj or gate/up_proj.
* ``sigmoid_gate(attn_out, gate)`` -> ``[B, T, H*D]``: drop-in for
  reference/d3_kernels.py:502-525 (``attn_out * sigmoid(gate)``, core.py:297).
* ``sigmoid_gate_quant(attn_out, gate, mode)`` -> ``(q, scale)``: the gated rows
  quantised for o_proj.

bf16 tensors on the GPU only; rows of up to 6144 elements (a multiple of 8),
16-byte aligned. A ``RuntimeError`` names any other case; there is no fallback.
"""

from __future__ import annotations

import torch

from .. import _lib
from .quant import _FP8, _mode_code


def _check_bf16(t: torch.Tensor, what: str) -> None:
    _lib.require_cuda(t, what)
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"{what}: expected bfloat16, got {t.dtype}")


def _rows(t: torch.Tensor, what: str) -> torch.Tensor:
    """[..., K] -> [M, K] view with unit last stride (copied only if it has none)."""
    flat = t.reshape(-1, t.shape[-1])
    if flat.stride(1) != 1 or flat.stride(0) < flat.shape[1]:
        flat = flat.contiguous()
    return flat


def _norm(residual, delta, weight_plus_one, eps, rowmask, mode_code):
    _check_bf16(residual, "add_rmsnorm")
    shape = residual.shape
    res = _rows(residual, "residual")
    M, K = res.shape
    dev = res.device
    d = None
    if delta is not None:
        _check_bf16(delta, "add_rmsnorm")
        if delta.shape != shape:
            raise RuntimeError(f"delta {tuple(delta.shape)} and residual {tuple(shape)} differ")
        d = _rows(delta, "delta")
    w1 = weight_plus_one.to(device=dev, dtype=torch.float32).contiguous()
    if w1.numel() != K:
        raise RuntimeError(f"weight_plus_one has {w1.numel()} elements for rows of {K}")
    mask = None
    if rowmask is not None:
        mask = rowmask.to(device=dev, dtype=torch.int32).reshape(-1).contiguous()
        if mask.numel() != M:
            raise RuntimeError(f"rowmask has {mask.numel()} entries for {M} rows")
    hidden = torch.empty((M, K), dtype=torch.bfloat16, device=dev) if d is not None else res
    normed = torch.empty((M, K), dtype=torch.bfloat16, device=dev) if mode_code == _lib.MODE_NONE else None
    q = scale = None
    if mode_code != _lib.MODE_NONE:
        q = torch.empty((M, K), dtype=_FP8 if mode_code == _lib.MODE_FP8 else torch.int8, device=dev)
        scale = torch.empty((M,), dtype=torch.float32, device=dev)
    if M:
        status = _lib.lib().d3b_add_rmsnorm_quant(
            _lib.ptr(res), res.stride(0), _lib.ptr(d), d.stride(0) if d is not None else 0, _lib.ptr(w1), float(eps),
            _lib.ptr(mask), _lib.ptr(hidden if d is not None else None), K, _lib.ptr(normed), K, _lib.ptr(q),
            _lib.ptr(scale), M, K, mode_code, _lib.stream_of(res),
        )
        _lib.check(status, "d3b_add_rmsnorm_quant")
    hidden_out = hidden.reshape(shape) if d is not None else residual
    return hidden_out, normed, q, scale


def add_rmsnorm(residual: torch.Tensor, delta: torch.Tensor | None, weight_plus_one: torch.Tensor, eps: float,
                rowmask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(hidden, normed) bf16: hidden = residual + delta (or residual), normed = Qwen3.5 RMSNorm of hidden.

    ``weight_plus_one`` is the fp32 ``1 + w``; ``rowmask`` (one integer per row)
    zeroes the normed rows of padding (reference/d3_kernels.py:145-170).
    """
    hidden, normed, _, _ = _norm(residual, delta, weight_plus_one, eps, rowmask, _lib.MODE_NONE)
    return hidden, normed.reshape(residual.shape)


def add_rmsnorm_quant(residual: torch.Tensor, delta: torch.Tensor | None, weight_plus_one: torch.Tensor, eps: float,
                      mode: str, rowmask: torch.Tensor | None = None):
    """(hidden, q [M, K], scale [M, 1]): the normed rows quantised per row in ``mode`` ("fp8"/"int8")."""
    hidden, _, q, scale = _norm(residual, delta, weight_plus_one, eps, rowmask, _mode_code(mode))
    return hidden, q, scale[:, None]


def _gate(attn_out, gate, mode_code):
    _check_bf16(attn_out, "sigmoid_gate")
    _check_bf16(gate, "sigmoid_gate")
    if attn_out.dim() != 4 or gate.shape != attn_out.shape:
        raise RuntimeError(f"attn_out and gate must both be [B, T, H, D], got {tuple(attn_out.shape)}, "
                           f"{tuple(gate.shape)}")
    if attn_out.stride(3) != 1:
        attn_out = attn_out.contiguous()
    if gate.stride(3) != 1:
        gate = gate.contiguous()
    B, T, H, D = attn_out.shape
    dev = attn_out.device
    gated = torch.empty((B, T, H * D), dtype=torch.bfloat16, device=dev) if mode_code == _lib.MODE_NONE else None
    q = scale = None
    if mode_code != _lib.MODE_NONE:
        q = torch.empty((B * T, H * D), dtype=_FP8 if mode_code == _lib.MODE_FP8 else torch.int8, device=dev)
        scale = torch.empty((B * T,), dtype=torch.float32, device=dev)
    if B * T:
        sa = _lib.i64_array(attn_out.stride()[:3])
        sg = _lib.i64_array(gate.stride()[:3])
        status = _lib.lib().d3b_sigmoid_gate_quant(
            _lib.ptr(attn_out), sa, _lib.ptr(gate), sg, _lib.ptr(gated), _lib.ptr(q), _lib.ptr(scale), B, T, H, D,
            mode_code, _lib.stream_of(attn_out),
        )
        _lib.check(status, "d3b_sigmoid_gate_quant")
    return gated, q, scale


def sigmoid_gate(attn_out: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """``attn_out * sigmoid(gate)`` -> [B, T, H * D] bf16 from [B, T, H, D] views with unit last stride."""
    gated, _, _ = _gate(attn_out, gate, _lib.MODE_NONE)
    return gated


def sigmoid_gate_quant(attn_out: torch.Tensor, gate: torch.Tensor, mode: str):
    """(q [B*T, H*D], scale [B*T, 1]): the gated rows quantised per row in ``mode`` for o_proj."""
    _, q, scale = _gate(attn_out, gate, _mode_code(mode))
    return q, scale[:, None]


def _out_buffers(M, K, mode_code, dev):
    out = torch.empty((M, K), dtype=torch.bfloat16, device=dev) if mode_code == _lib.MODE_NONE else None
    q = scale = None
    if mode_code != _lib.MODE_NONE:
        q = torch.empty((M, K), dtype=_FP8 if mode_code == _lib.MODE_FP8 else torch.int8, device=dev)
        scale = torch.empty((M,), dtype=torch.float32, device=dev)
    return out, q, scale


def _silu_mul(gate_up: torch.Tensor, mode_code: int):
    _check_bf16(gate_up, "silu_mul")
    rows = _rows(gate_up, "gate_up")
    M, two_i = rows.shape
    if two_i % 2:
        raise RuntimeError("gate_up rows must hold gate and up halves")
    out, q, scale = _out_buffers(M, two_i // 2, mode_code, rows.device)
    if M:
        st = _lib.lib().d3b_silu_mul_quant(_lib.ptr(rows), rows.stride(0), _lib.ptr(out), _lib.ptr(q), _lib.ptr(scale),
                                          M, two_i // 2, mode_code, _lib.stream_of(rows))
        _lib.check(st, "d3b_silu_mul_quant")
    return out, q, scale


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(silu(gate)) * up) [M, I] from the fused gate/up projection's rows [M, 2I]
    (the Qwen3.5 MLP's act_fn(gate_proj(x)) * up_proj(x))."""
    out, _, _ = _silu_mul(gate_up, _lib.MODE_NONE)
    return out


def silu_mul_quant(gate_up: torch.Tensor, mode: str):
    """(q [M, I], scale [M, 1]): the MLP activation quantised per row for down_proj."""
    _, q, scale = _silu_mul(gate_up, _mode_code(mode))
    return q, scale[:, None]


def _gated_norm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float, head_dim: int, mode_code: int):
    _check_bf16(x, "gated_rmsnorm")
    _check_bf16(z, "gated_rmsnorm")
    xr, zr = _rows(x, "x"), _rows(z, "z")
    if xr.shape != zr.shape:
        raise RuntimeError(f"x {tuple(xr.shape)} and z {tuple(zr.shape)} differ")
    M, K = xr.shape
    w = weight.to(device=xr.device, dtype=torch.bfloat16).contiguous()
    if w.numel() != head_dim:
        raise RuntimeError(f"weight has {w.numel()} values for head_dim {head_dim}")
    out, q, scale = _out_buffers(M, K, mode_code, xr.device)
    if M:
        st = _lib.lib().d3b_gated_rmsnorm_quant(_lib.ptr(xr), xr.stride(0), _lib.ptr(zr), zr.stride(0), _lib.ptr(w),
                                               float(eps), head_dim, _lib.ptr(out), _lib.ptr(q), _lib.ptr(scale), M, K,
                                               mode_code, _lib.stream_of(xr))
        _lib.check(st, "d3b_gated_rmsnorm_quant")
    return out, q, scale


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float, head_dim: int) -> torch.Tensor:
    """Qwen3_5RMSNormGated over heads of ``head_dim`` on token rows x, z [..., K] -> [M, K] bf16."""
    out, _, _ = _gated_norm(x, z, weight, eps, head_dim, _lib.MODE_NONE)
    return out


def gated_rmsnorm_quant(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float, head_dim: int,
                        mode: str):
    """(q [M, K], scale [M, 1]): the gated norm's token rows quantised for out_proj."""
    _, q, scale = _gated_norm(x, z, weight, eps, head_dim, _mode_code(mode))
    return q, scale[:, None]


def qk_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 eps: float) -> torch.Tensor:
    """q_norm / k_norm (Qwen3_5RMSNorm per head) then the partial rotary embedding, one pass.

    x [rows, T, heads, 128] bf16 (any row/token/head strides, last dim contiguous), weight
    [128] (the norm's raw weight; the kernel applies 1 + w), cos/sin [rows, T, rd] bf16.
    Returns [rows, T, heads, 128] bf16, token-major; ``.transpose(1, 2)`` gives the
    [rows, heads, T, 128] view the attention kernels read (d3trt/model/core.py:233-237).
    """
    _check_bf16(x, "qk_norm_rope")
    if x.dim() != 4 or x.stride(-1) != 1:
        raise RuntimeError(f"qk_norm_rope: x must be [rows, T, heads, D] with a contiguous last dim, got "
                           f"{tuple(x.shape)} strides {x.stride()}")
    rows, T, heads, D = x.shape
    if cos.shape != sin.shape or cos.dim() != 3 or tuple(cos.shape[:2]) != (rows, T):
        raise RuntimeError(f"qk_norm_rope: cos/sin must be [rows, T, rd], got {tuple(cos.shape)}, {tuple(sin.shape)}")
    cos = cos.to(torch.bfloat16)
    sin = sin.to(torch.bfloat16)
    if cos.stride(-1) != 1 or cos.stride() != sin.stride():
        cos, sin = cos.contiguous(), sin.contiguous()
    w = weight.to(device=x.device, dtype=torch.bfloat16).contiguous()
    out = torch.empty(rows, T, heads, D, dtype=torch.bfloat16, device=x.device)
    st = _lib.lib().d3b_qk_norm_rope(
        _lib.ptr(x), _lib.i64_array(x.stride()[:3]), _lib.ptr(w), _lib.ptr(cos), _lib.ptr(sin),
        _lib.i64_array(cos.stride()[:2]), _lib.ptr(out), rows, T, heads, D, int(cos.shape[-1]), float(eps),
        _lib.stream_of(x))
    _lib.check(st, "d3b_qk_norm_rope")
    return out


def gdn_gates(a: torch.Tensor, b: torch.Tensor, neg_exp_a: torch.Tensor, dt_bias: torch.Tensor):
    """(g [M, HV] fp32, beta [M, HV] bf16) of the Gated DeltaNet layer, one kernel:
    beta = b.sigmoid(), g = neg_exp_a * softplus(a.float() + dt_bias) with neg_exp_a =
    -exp(A_log.float()) and dt_bias fp32 per value head (d3trt/model/core.py:341-342).
    a, b: [M, HV] bf16 (row slices of the input projection are read in place)."""
    _check_bf16(a, "gdn_gates")
    _check_bf16(b, "gdn_gates")
    if a.dim() != 2 or a.shape != b.shape or a.stride(1) != 1 or b.stride(1) != 1:
        raise RuntimeError(f"gdn_gates: a and b must be [M, HV] rows with a contiguous last dim, got "
                           f"{tuple(a.shape)} {a.stride()} and {tuple(b.shape)} {b.stride()}")
    M, HV = a.shape
    ne = neg_exp_a.to(device=a.device, dtype=torch.float32).contiguous()
    dtb = dt_bias.to(device=a.device, dtype=torch.float32).contiguous()
    if ne.numel() != HV or dtb.numel() != HV:
        raise RuntimeError(f"gdn_gates: {HV} value heads, got {ne.numel()} and {dtb.numel()} per-head values")
    g = torch.empty(M, HV, dtype=torch.float32, device=a.device)
    beta = torch.empty(M, HV, dtype=torch.bfloat16, device=a.device)
    st = _lib.lib().d3b_gdn_gates(_lib.ptr(a), max(a.stride(0), HV), _lib.ptr(b), max(b.stride(0), HV), _lib.ptr(ne),
                                  _lib.ptr(dtb), _lib.ptr(g), _lib.ptr(beta), M, HV, _lib.stream_of(a))
    _lib.check(st, "d3b_gdn_gates")
    return g, beta
