"""Readout oracle (numpy, float32) — test infrastructure only.

Restates the probabilities body of d3trt/model/trtllm_stack.py:459-468
(identical to hf_stack.py:67-84 and reference/d3_runtime.py:2820-2829):
    logits = f32(hidden) @ R^T ; logits[b, j >= counts[b]] = -inf ;
    probs = softmax(logits / T) ; rows cut to counts[b]
"""

from __future__ import annotations

from typing import Sequence

import numpy as np


def probabilities(hidden: np.ndarray, readout: np.ndarray, counts: Sequence[int], temperature: float) -> np.ndarray:
    """-> [B, n_opt] float32 (full rows, masked entries 0)."""
    h = np.asarray(hidden, dtype=np.float32).astype(np.float64)
    r = np.asarray(readout, dtype=np.float32).astype(np.float64)
    logits = (h @ r.T).astype(np.float32)
    n_opt = r.shape[0]
    mask = np.arange(n_opt)[None, :] >= np.asarray(counts)[:, None]
    logits = np.where(mask, -np.inf, logits).astype(np.float32)
    z = (logits / np.float32(temperature)).astype(np.float64)
    z = z - z.max(axis=1, keepdims=True)
    e = np.exp(z)
    return (e / e.sum(axis=1, keepdims=True)).astype(np.float32)


def probabilities_lists(hidden, readout, counts, temperature) -> list[list[float]]:
    probs = probabilities(hidden, readout, counts, temperature)
    return [row[: int(c)].tolist() for row, c in zip(probs, counts)]
