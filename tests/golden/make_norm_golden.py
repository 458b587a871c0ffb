"""Generate tests/golden/norm_quant.npz by running the model's own modules.

    python tests/golden/make_norm_golden.py --reference <path to a d3-turbo-trt checkout>

(or set D3_REFERENCE_DIR). Records, on seeded bf16 inputs, what the reference's
eager forward computes for the two producers of every QuantLinear input:

* add + RMSNorm: ``hidden = residual + delta`` in bf16 (d3trt/model/core.py:219,
  ``hidden = residual + mixed``), then transformers' ``Qwen3_5RMSNorm``
  (modeling_qwen3_5.py, the layer the reference's HF stack runs as
  ``input_layernorm`` / ``post_attention_layernorm``) with a seeded weight.
* sigmoid gate: ``out * torch.sigmoid(gate)`` in bf16 (core.py:297).

and the reference's ``quantize_rows`` (d3trt/model/quant.py:92-100) of both
outputs in fp8 and int8. The fixture is committed; this script is only needed
to regenerate it.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def codes(q: torch.Tensor) -> np.ndarray:
    return q.view(torch.uint8).numpy() if q.dtype != torch.int8 else q.numpy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("D3_REFERENCE_DIR"))
    args = ap.parse_args()
    if not args.reference or not Path(args.reference, "d3trt").is_dir():
        raise SystemExit("pass --reference <d3-turbo-trt checkout> (or set D3_REFERENCE_DIR)")
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from d3trt.model import quant  # noqa: E402
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNorm  # noqa: E402

    torch.set_grad_enabled(False)
    g = torch.Generator().manual_seed(7)
    M, K, eps = 32, 1024, 1e-6
    residual = torch.randn(M, K, generator=g).to(torch.bfloat16)
    delta = (torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16)
    delta[3] *= 40.0  # a row with a large residual update
    norm = Qwen3_5RMSNorm(K, eps=eps)
    norm.weight.copy_(torch.randn(K, generator=g) * 0.1)
    hidden = residual + delta
    normed = norm(hidden)
    out: dict[str, np.ndarray] = {
        "residual": bf16_bits(residual), "delta": bf16_bits(delta), "weight": norm.weight.numpy(),
        "eps": np.float64(eps), "hidden": bf16_bits(hidden), "normed": bf16_bits(normed),
    }
    # attention output and gate, [B, T, H, D] as core.py:295-297 sees them
    attn = torch.randn(2, 8, 4, 64, generator=g).to(torch.bfloat16)
    gate = (torch.randn(2, 8, 4, 64, generator=g) * 3.0).to(torch.bfloat16)
    gated = (attn.reshape(16, 256) * torch.sigmoid(gate.reshape(16, 256)))
    out.update(attn=bf16_bits(attn), gate=bf16_bits(gate), gated=bf16_bits(gated))
    for mode in ("fp8", "int8"):
        q, s = quant.quantize_rows(normed, mode)
        out[f"normed_q_{mode}"], out[f"normed_s_{mode}"] = codes(q), s.numpy()
        q, s = quant.quantize_rows(gated, mode)
        out[f"gated_q_{mode}"], out[f"gated_s_{mode}"] = codes(q), s.numpy()
    np.savez_compressed(OUT / "norm_quant.npz", **out)
    print("norm_quant.npz", (OUT / "norm_quant.npz").stat().st_size)


if __name__ == "__main__":
    main()
