"""Generate the golden vectors under tests/golden/ by running the reference itself.

    python tests/golden/make_golden.py --reference <path to a d3-turbo-trt checkout>

(or set D3_REFERENCE_DIR). Imports the reference's own functions and records
their outputs on seeded inputs:

* quant.npz   — d3trt.model.quant.quantize_rows / quantize_weight and
                QuantLinear._emulated (quant.py:77-100, :158-162), plus the exact
                int32 accumulators (q.float() @ w.float().t(), exact here).
* attn_cfg1.npz: a 512-token state + 8 blocks of 32 tokens,
                H=8, H_kv=2, D=64, Q/K/V ~ N(0,1) rounded to bf16, scale 1/8.
                State rows from d3trt.model.ops.sdpa_state (ops.py:107-124),
                question rows from ops.sdpa_questions (ops.py:127-171), checked
                here against one dense masked SDPA built like
                reference/d3_runtime.py:1396-1400.
* attn_ragged.npz — small ragged cases (empty and length-1 blocks, H/H_kv that
                does not divide 128, D = 32 / 64 / 256) through ops.sdpa_questions.
* readout.npz — the probabilities body of TrtllmStack (trtllm_stack.py:451-468).

Inputs are bf16-representable; the reference is run in float32 on the CPU.
The fixtures are committed; this script is only needed to regenerate them.
"""

from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

OUT = Path(__file__).resolve().parent


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def bf16_values(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


def make_quant(quant) -> None:
    g = torch.Generator().manual_seed(0)
    out: dict[str, np.ndarray] = {}
    # activations: 64 x 320 bf16, 1% of channels x20, one zero row, one x1000 row
    x = torch.randn(64, 320, generator=g)
    cols = torch.randperm(320, generator=g)[:4]
    x[:, cols] *= 20.0
    x[5] = 0.0
    x[9] *= 1000.0
    x = x.to(torch.bfloat16)
    out["rows_x_bf16"] = bf16_bits(x)
    for mode in ("fp8", "int8"):
        q, s = quant.quantize_rows(x, mode)
        out[f"rows_q_{mode}"] = q.view(torch.uint8).numpy() if mode == "fp8" else q.numpy()
        out[f"rows_s_{mode}"] = s.numpy()
    # fp32 activations with a ragged K (no 16-byte vector path)
    x32 = torch.randn(16, 200, generator=g) * 3.0
    out["rows_x_f32"] = x32.numpy()
    for mode in ("fp8", "int8"):
        q, s = quant.quantize_rows(x32, mode)
        out[f"rows32_q_{mode}"] = q.view(torch.uint8).numpy() if mode == "fp8" else q.numpy()
        out[f"rows32_s_{mode}"] = s.numpy()
    # weights: [96, 256] * 0.02 (tests/test_quant.py:18)
    w = (torch.randn(96, 256, generator=g) * 0.02).to(torch.bfloat16)
    out["w_bf16"] = bf16_bits(w)
    for mode in ("fp8", "int8"):
        q, s = quant.quantize_weight(w, mode)
        out[f"w_q_{mode}"] = q.view(torch.uint8).numpy() if mode == "fp8" else q.numpy()
        out[f"w_s_{mode}"] = s.numpy()
    # QuantLinear._emulated on x [3, 5, 256] bf16 (tests/test_quant.py:15-26)
    xl = torch.randn(3, 5, 256, generator=g).to(torch.bfloat16)
    out["lin_x_bf16"] = bf16_bits(xl)
    for mode in ("fp8", "int8"):
        layer = quant.QuantLinear(256, 96, mode=mode, dtype=torch.bfloat16, device="cpu")
        layer.load_full(w)
        y = layer(xl)
        assert layer.kernel == "emulated"
        out[f"lin_y_{mode}_bf16"] = bf16_bits(y)
        qa, sa = quant.quantize_rows(xl.reshape(-1, 256), mode)
        acc = qa.float() @ layer.weight.float().t()
        out[f"lin_acc_{mode}"] = acc.numpy()
        out[f"lin_f32_{mode}"] = (acc * sa * layer.weight_scale[None, :]).numpy()
    np.savez_compressed(OUT / "quant.npz", **out)


def make_cfg1(ops) -> None:
    g = torch.Generator().manual_seed(1)
    state, nb, lq, heads, kv_heads, dim = 512, 8, 32, 8, 2, 64
    total = state + nb * lq
    scale = 1.0 / 8.0
    Q = bf16_values(torch.randn(total, heads, dim, generator=g))
    K = bf16_values(torch.randn(total, kv_heads, dim, generator=g))
    V = bf16_values(torch.randn(total, kv_heads, dim, generator=g))
    # state rows: ops.sdpa_state on [1, H, S, D]
    qs = Q[:state].transpose(0, 1)[None]
    ks = K[:state].transpose(0, 1)[None]
    vs = V[:state].transpose(0, 1)[None]
    out_state = ops.sdpa_state(qs, ks, vs, scale=scale)[0].transpose(0, 1)
    # question rows: ops.sdpa_questions on [B, H, L, D] with [H_kv, S, D] state
    qq = Q[state:].view(nb, lq, heads, dim).permute(0, 2, 1, 3)
    kq = K[state:].view(nb, lq, kv_heads, dim).permute(0, 2, 1, 3)
    vq = V[state:].view(nb, lq, kv_heads, dim).permute(0, 2, 1, 3)
    out_q = ops.sdpa_questions(qq, ks[0], vs[0], kq, vq, [lq] * nb, scale=scale)
    out = torch.cat([out_state, out_q.permute(0, 2, 1, 3).reshape(nb * lq, heads, dim)], dim=0)
    # cross-check against one dense masked SDPA (d3_runtime.py:1396-1400 semantics)
    allowed = torch.zeros(total, total, dtype=torch.bool)
    allowed[:state, :state] = True
    for i in range(nb):
        a, b = state + i * lq, state + (i + 1) * lq
        allowed[a:b, :state] = True
        allowed[a:b, a:b] = True
    dense = F.scaled_dot_product_attention(
        Q.transpose(0, 1)[None], K.transpose(0, 1).repeat_interleave(heads // kv_heads, 0)[None],
        V.transpose(0, 1).repeat_interleave(heads // kv_heads, 0)[None], attn_mask=allowed, scale=scale,
    )[0].transpose(0, 1)
    assert torch.allclose(dense, out, atol=1e-5), float((dense - out).abs().max())
    np.savez_compressed(
        OUT / "attn_cfg1.npz",
        Q=bf16_bits(Q), K=bf16_bits(K), V=bf16_bits(V), out=out.numpy(),
        meta=np.array([state, nb, lq, heads, kv_heads, dim], dtype=np.int64), scale=np.float64(scale),
    )


def make_ragged(ops) -> None:
    g = torch.Generator().manual_seed(2)
    cases = {
        # name: (B, H, H_kv, L, D, S, lengths)
        "d32_g2": (5, 4, 2, 24, 32, 96, [24, 1, 0, 13, 24]),
        "d64_g3": (3, 6, 2, 20, 64, 130, [20, 7, 19]),
        "d256_g1": (2, 2, 2, 9, 256, 70, [9, 4]),
        "d128_g8": (2, 16, 2, 20, 128, 150, [20, 3]),
    }
    out: dict[str, np.ndarray] = {}
    for name, (B, H, Hkv, L, D, S, lens) in cases.items():
        scale = D**-0.5
        q = bf16_values(torch.randn(B, H, L, D, generator=g))
        ks = bf16_values(torch.randn(Hkv, S, D, generator=g))
        vs = bf16_values(torch.randn(Hkv, S, D, generator=g))
        kq = bf16_values(torch.randn(B, Hkv, L, D, generator=g))
        vq = bf16_values(torch.randn(B, Hkv, L, D, generator=g))
        o = ops.sdpa_questions(q, ks, vs, kq, vq, lens, scale=scale)
        for key, val in (("q", q), ("ks", ks), ("vs", vs), ("kq", kq), ("vq", vq)):
            out[f"{name}_{key}"] = bf16_bits(val)
        out[f"{name}_lens"] = np.array(lens, dtype=np.int32)
        out[f"{name}_out"] = o.numpy()
        out[f"{name}_scale"] = np.float64(scale)
    np.savez_compressed(OUT / "attn_ragged.npz", **out)


def make_readout(stack_mod) -> None:
    g = torch.Generator().manual_seed(3)
    rows, k, n_opt = 12, 256, 255
    hidden = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    readout = torch.randn(n_opt, k, generator=g) * 0.02 * 8.0
    counts = [255, 1, 2, 7, 100, 254, 255, 3, 64, 128, 200, 17]
    fake = types.SimpleNamespace(readout=readout, max_options=n_opt)
    out: dict[str, np.ndarray] = {"hidden_bf16": bf16_bits(hidden), "readout": readout.numpy(),
                                  "counts": np.array(counts, dtype=np.int32)}
    for tag, temp in (("t1", 1.0), ("t07", 0.7)):
        lists = stack_mod.TrtllmStack.probabilities(fake, hidden, counts, temperature=temp)
        full = np.zeros((rows, n_opt), dtype=np.float32)
        for i, row in enumerate(lists):
            full[i, : len(row)] = row
        out[f"probs_{tag}"] = full
        out[f"temp_{tag}"] = np.float64(temp)
    np.savez_compressed(OUT / "readout.npz", **out)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("D3_REFERENCE_DIR"))
    args = ap.parse_args()
    if not args.reference or not Path(args.reference, "d3trt").is_dir():
        raise SystemExit("pass --reference <d3-turbo-trt checkout> (or set D3_REFERENCE_DIR)")
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from d3trt.model import ops, quant, trtllm_stack  # noqa: E402

    torch.set_grad_enabled(False)
    make_quant(quant)
    make_cfg1(ops)
    make_ragged(ops)
    make_readout(trtllm_stack)
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
