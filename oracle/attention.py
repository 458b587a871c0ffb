"""Prefix-bidirectional attention oracle (torch on the CPU) — test infrastructure only.

Restates:
* ops.sdpa_questions (d3trt/model/ops.py:127-171): per question block b, the
  queries of its first lengths[b] tokens attend to cat(state keys, own keys
  [:lengths[b]]) with GQA (kv head = h // (H/H_kv), prefix_bidir.py:85);
  padding rows are zero.
* ops.sdpa_state (ops.py:107-124): dense non-causal GQA attention over the state.
* StateOnce._attention mask semantics (reference/d3_runtime.py:1378-1407,
  mask at :1396-1400) as one dense masked pass over [state | blocks].
The softmax is written out (max-subtracted exp, sum, divide) in float64 by
default, or float32 for the timed CPU baseline.
"""

from __future__ import annotations

from typing import Sequence

import torch


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """q [G, Lq, D] (one kv group), k/v [Lk, D] -> [G, Lq, D]."""
    s = torch.matmul(q, k.transpose(0, 1)) * scale
    s = s - s.amax(dim=-1, keepdim=True)
    p = torch.exp(s)
    p = p / p.sum(dim=-1, keepdim=True)
    return torch.matmul(p, v)


def questions(
    q: torch.Tensor,
    k_state: torch.Tensor,
    v_state: torch.Tensor,
    k_q: torch.Tensor,
    v_q: torch.Tensor,
    lengths: Sequence[int],
    scale: float,
    dtype: torch.dtype = torch.float64,
) -> torch.Tensor:
    """[B,H,L,D] question pass over [H_kv,S,D] state + own block (ops.py:127-171)."""
    rows, heads, width, dim = q.shape
    kv_heads = k_state.shape[0]
    groups = heads // kv_heads
    q, k_state, v_state, k_q, v_q = (t.to(dtype) for t in (q, k_state, v_state, k_q, v_q))
    out = torch.zeros((rows, heads, width, dim), dtype=dtype)
    for b in range(rows):
        n = int(lengths[b])
        if n == 0:
            continue
        for g in range(kv_heads):
            keys = torch.cat([k_state[g], k_q[b, g, :n]], dim=0)
            vals = torch.cat([v_state[g], v_q[b, g, :n]], dim=0)
            hs = slice(g * groups, (g + 1) * groups)
            out[b, hs, :n] = _attend(q[b, hs, :n], keys, vals, scale)
    return out


def questions_sdpa(
    q: torch.Tensor,
    k_state: torch.Tensor,
    v_state: torch.Tensor,
    k_q: torch.Tensor,
    v_q: torch.Tensor,
    lengths: Sequence[int],
    scale: float,
) -> torch.Tensor:
    """The question pass as the reference's CPU path computes it (ops.sdpa_questions,
    d3trt/model/ops.py:127-171): per block, one torch scaled_dot_product_attention call
    over cat(state keys, own keys[:length]) with native GQA, in the inputs' dtype. The
    timed reference arm and CPU baseline run this, so they use the same torch CPU kernel
    as the reference; padding rows are zero."""
    import torch.nn.functional as F

    out = q.new_zeros(q.shape)
    for b in range(q.shape[0]):
        n = int(lengths[b])
        if n == 0:
            continue
        keys = torch.cat([k_state, k_q[b, :, :n]], dim=1)
        vals = torch.cat([v_state, v_q[b, :, :n]], dim=1)
        out[b, :, :n] = F.scaled_dot_product_attention(q[b, :, :n][None], keys[None], vals[None], scale=scale,
                                                      enable_gqa=True)[0]
    return out


def state(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, dtype: torch.dtype = torch.float64):
    """[B,H,S,D] dense bidirectional GQA attention over [B,H_kv,S,D] (ops.py:107-124)."""
    rows, heads, tokens, dim = q.shape
    kv_heads = k.shape[1]
    groups = heads // kv_heads
    q, k, v = (t.to(dtype) for t in (q, k, v))
    out = torch.empty((rows, heads, tokens, dim), dtype=dtype)
    for b in range(rows):
        for g in range(kv_heads):
            hs = slice(g * groups, (g + 1) * groups)
            out[b, hs] = _attend(q[b, hs], k[b, g], v[b, g], scale)
    return out


def masked_sequence(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state_len: int, block_lens: Sequence[int], scale: float
) -> torch.Tensor:
    """One dense masked pass over a [state | block_0 | block_1 | ...] sequence.

    q [T, H, D], k/v [T, H_kv, D] with T = state_len + sum(block_lens). State
    tokens see all state tokens; block i's tokens see all state tokens and
    block i, bidirectionally (reference/d3_runtime.py:1396-1400).
    """
    total, heads, dim = q.shape
    kv_heads = k.shape[1]
    groups = heads // kv_heads
    allowed = torch.zeros((total, total), dtype=torch.bool)
    allowed[:state_len, :state_len] = True
    start = state_len
    for n in block_lens:
        allowed[start : start + n, :state_len] = True
        allowed[start : start + n, start : start + n] = True
        start += n
    qd, kd, vd = (t.to(torch.float64) for t in (q, k, v))
    out = torch.empty((total, heads, dim), dtype=torch.float64)
    for h in range(heads):
        g = h // groups
        s = (qd[:, h] @ kd[:, g].T) * scale
        s = s.masked_fill(~allowed, float("-inf"))
        s = s - s.amax(dim=-1, keepdim=True)
        p = torch.exp(s)
        p = p / p.sum(dim=-1, keepdim=True)
        out[:, h] = p @ vd[:, g]
    return out
