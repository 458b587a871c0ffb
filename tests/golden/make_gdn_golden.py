"""Record the reference's gated delta rule outputs as golden vectors.

    python tests/golden/make_gdn_golden.py --reference <path to a d3-turbo-trt checkout>

(or set D3_REFERENCE_DIR). Calls d3trt.model.ops.recurrent_gated_delta_rule and
ops.chunk_gated_delta_rule (ops.py:287-360) on the CPU, where they run the reference's
fallback (transformers' torch_recurrent_gated_delta_rule / torch_chunk_gated_delta_rule),
with q/k repeated from H to HV heads as D3Core does (core.py:345-347) and
use_qk_l2norm_in_kernel=True. Inputs are seeded, bf16-representable, passed in float32;
g is a log decay built like core.py:341 (-exp(A_log) * softplus(a + dt_bias)), beta a
sigmoid. Writes gdn.npz (inputs as bf16 bits, outputs of both reference paths).
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent

# name: (B, T, H, HV, K, V, initial state shared across rows?)
CASES = {
    "k64": (2, 37, 1, 2, 64, 64, True),
    "k128": (1, 9, 1, 1, 128, 128, True),
    "zero_init": (2, 5, 2, 2, 64, 64, None),
}


def bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("D3_REFERENCE_DIR"))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference or set D3_REFERENCE_DIR")
    sys.path.insert(0, args.reference)
    from d3trt.model import ops

    out = {}
    for i, (name, (B, T, H, HV, K, V, shared)) in enumerate(CASES.items()):
        gen = torch.Generator().manual_seed(100 + i)
        q = bf16(torch.randn(B, T, H, K, generator=gen))
        k = bf16(torch.randn(B, T, H, K, generator=gen))
        v = bf16(torch.randn(B, T, HV, V, generator=gen))
        a = torch.randn(B, T, HV, generator=gen)
        a_log = torch.rand(HV, generator=gen) * 2 - 1
        dt_bias = torch.randn(HV, generator=gen) * 0.5
        g = -a_log.exp() * F.softplus(a + dt_bias)
        beta = bf16(torch.sigmoid(torch.randn(B, T, HV, generator=gen)))
        h0 = torch.randn(1, HV, K, V, generator=gen) * 0.5 if shared else None
        rep = HV // H
        qr, kr = q.repeat_interleave(rep, dim=2), k.repeat_interleave(rep, dim=2)
        init = None if h0 is None else h0.expand(B, -1, -1, -1).contiguous()
        o_rec, s_rec = ops.recurrent_gated_delta_rule(qr, kr, v, g=g, beta=beta, initial_state=init,
                                                      output_final_state=True, use_qk_l2norm_in_kernel=True)
        o_chk, s_chk = ops.chunk_gated_delta_rule(qr, kr, v, g=g, beta=beta, initial_state=init,
                                                  output_final_state=True, use_qk_l2norm_in_kernel=True)
        out[f"{name}_meta"] = np.array([B, T, H, HV, K, V])
        for key, t in (("q", q), ("k", k), ("v", v), ("beta", beta)):
            out[f"{name}_{key}"] = t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        out[f"{name}_g"] = g.numpy().astype(np.float32)
        if h0 is not None:
            out[f"{name}_h0"] = h0[0].numpy().astype(np.float32)
        out[f"{name}_o_rec"] = o_rec.float().numpy()
        out[f"{name}_s_rec"] = s_rec.float().numpy()
        out[f"{name}_o_chunk"] = o_chk.float().numpy()
        out[f"{name}_s_chunk"] = s_chk.float().numpy()
    np.savez_compressed(HERE / "gdn.npz", **out)
    print(sorted(out))


if __name__ == "__main__":
    main()
