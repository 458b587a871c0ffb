"""The GDN layers' causal depthwise convolution + SiLU on token-major rows (drop-in for
the math of d3trt/model/ops.py:266-285 as D3Core uses it, core.py:311-330).

``causal_conv1d_silu(x, weight, tail=None)``: ``x`` [B, T, C] bf16 as the in_proj GEMM
writes it (channels contiguous; any row and token strides that are multiples of 8),
``weight`` [C, W], ``tail`` the snapshot's last W-1 inputs ``[1 or B, C, W-1]`` (any
strides) or None for the state pass. Returns [B, T, C] bf16. Equivalent to the
reference's ``F.silu(F.conv1d(cat([tail, x^T]), weight, groups=C, padding=W-1))``
restricted to the new tokens, with no transpose and no concatenation.
"""

from __future__ import annotations

import torch

from .. import _lib


def causal_conv1d_silu(x: torch.Tensor, weight: torch.Tensor, tail: torch.Tensor | None = None) -> torch.Tensor:
    _lib.require_cuda(x, "causal_conv1d_silu")
    if x.dtype != torch.bfloat16 or x.dim() != 3:
        raise RuntimeError("causal_conv1d_silu: x must be [B, T, C] bf16")
    B, T, C = x.shape
    if weight.dim() == 3:
        weight = weight.squeeze(1)
    if weight.shape[0] != C:
        raise RuntimeError(f"causal_conv1d_silu: weight {tuple(weight.shape)} for {C} channels")
    W = weight.shape[1]
    w = weight.to(device=x.device, dtype=torch.bfloat16).contiguous()
    if x.stride(2) != 1 or x.stride(0) % 8 or x.stride(1) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    st = None
    if tail is not None:
        if tail.dim() != 3 or tail.shape[1] != C or tail.shape[2] != W - 1 or tail.shape[0] not in (1, B):
            raise RuntimeError(f"causal_conv1d_silu: tail must be [1 or {B}, {C}, {W - 1}], got {tuple(tail.shape)}")
        if tail.dtype != torch.bfloat16:
            tail = tail.to(torch.bfloat16)
        st = _lib.i64_array([0 if tail.shape[0] == 1 else tail.stride(0), tail.stride(1), tail.stride(2)])
    out = torch.empty((B, T, C), dtype=torch.bfloat16, device=x.device)
    status = _lib.lib().d3b_causal_conv1d_silu(
        _lib.ptr(x), _lib.i64_array([x.stride(0), x.stride(1)]), _lib.ptr(tail), st, _lib.ptr(w), _lib.ptr(out),
        B, T, C, W, _lib.stream_of(x))
    _lib.check(status, "d3b_causal_conv1d_silu")
    return out
