"""Attention dispatch for the full-attention layers (drop-in for the attention half of
d3trt/model/ops.py).

The reference picks Triton, then FlashAttention, then SDPA and swallows any
exception on the way (ops.py:227-259). Here there is one path — the sm_100a
kernel — and a failure raises. ``return_kernel=True`` reports ``"sm100a"`` so
``CoreStats.attention_question`` (core.py:265) records what ran.
The Gated-DeltaNet half of the reference module is not on this path.
"""

from __future__ import annotations

from typing import Any, Sequence

import torch

from ..kernels.prefix_bidir import KERNEL_NAME, kernel_available, prefix_bidir_attention, state_attention

_REPORT: dict[str, str] = {}


def kernel_report() -> dict[str, str]:
    """Which kernels serve the attention calls (reference: ops.py:29-30)."""
    _REPORT["prefix_bidir"] = KERNEL_NAME if kernel_available() else "missing"
    _REPORT["state_attention"] = _REPORT["prefix_bidir"]
    return dict(_REPORT)


def question_attention(
    q: torch.Tensor,
    k_state: torch.Tensor,
    v_state: torch.Tensor,
    k_q: torch.Tensor,
    v_q: torch.Tensor,
    lengths: Sequence[int],
    *,
    scale: float,
    prefer_triton: bool = True,
    return_kernel: bool = False,
) -> Any:
    """Shared-prefix question attention (reference signature: ops.py:227-259).

    ``prefer_triton`` is accepted for call compatibility and ignored: the sm_100a
    kernel is the only implementation.
    """
    del prefer_triton
    out = prefix_bidir_attention(q, k_state, v_state, k_q, v_q, lengths, scale=scale)
    return (out, KERNEL_NAME) if return_kernel else out


def flash_state(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float) -> torch.Tensor:
    """Bidirectional attention over one state block (reference: ops.py:174-193)."""
    return state_attention(q, k, v, scale=scale)


def sdpa_state(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float) -> torch.Tensor:
    """Same as :func:`flash_state` (reference name: ops.py:107-124)."""
    return state_attention(q, k, v, scale=scale)
