"""Gated delta rule oracle (numpy, fp64) — test infrastructure only.

The GDN layers' scan as the reference runs it: d3trt/model/core.py:333-372 builds
q, k (repeated from H to HV heads, :345-347), v, g = -exp(A_log) * softplus(a + dt_bias),
beta = sigmoid(b), and calls ops.recurrent_gated_delta_rule / chunk_gated_delta_rule
(d3trt/model/ops.py:287-360) with use_qk_l2norm_in_kernel=True. Those dispatch to
flash-linear-attention 0.5.1 on the GPU (a third-party package, not in the reference
tree) and to transformers' torch_recurrent_gated_delta_rule /
torch_chunk_gated_delta_rule on the CPU. The published algorithm (gated delta rule,
token-recurrent form), restated here in fp64:

    q, k <- x / sqrt(sum(x^2) + 1e-6)     (per token and head, when l2norm)
    q <- q * scale                         (scale = K^-1/2 by default)
    S <- exp(g_t) * S
    v' = beta_t * (v_t - S^T k_t)
    S <- S + k_t v'^T
    o_t = S^T q_t

with S [K, V] per (row, value head), S_0 = initial_state (zeros when absent). The q/k head
of value head hv is hv // (HV // H), which is what the reference's repeat_interleave builds.
Pinned against the reference's own CPU paths by tests/golden/make_gdn_golden.py.
"""

from __future__ import annotations

import numpy as np


def gated_delta_rule(q, k, v, g, beta, h0=None, scale=None, l2norm=True):
    """q, k [B,T,H,K]; v [B,T,HV,V]; g, beta [B,T,HV]; h0 [B,HV,K,V] or None -> (o [B,T,HV,V], S_T [B,HV,K,V])."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    g = np.asarray(g, np.float64)
    beta = np.asarray(beta, np.float64)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    rep = HV // H
    q = np.repeat(q, rep, axis=2)
    k = np.repeat(k, rep, axis=2)
    if l2norm:
        q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6)
        k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    q = q * (K ** -0.5 if scale is None else scale)
    S = np.zeros((B, HV, K, V)) if h0 is None else np.array(np.broadcast_to(h0, (B, HV, K, V)), np.float64)
    o = np.zeros((B, T, HV, V))
    for t in range(T):
        S = S * np.exp(g[:, t])[:, :, None, None]
        kv = np.einsum("bhk,bhkv->bhv", k[:, t], S)
        vn = beta[:, t][:, :, None] * (v[:, t] - kv)
        S = S + k[:, t][:, :, :, None] * vn[:, :, None, :]
        o[:, t] = np.einsum("bhk,bhkv->bhv", q[:, t], S)
    return o, S
