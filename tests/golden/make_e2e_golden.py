"""Generate tests/golden/e2e_4layer.npz by running the reference's own D3Core.

    python tests/golden/make_e2e_golden.py --reference <path to a d3-turbo-trt checkout>

(or set D3_REFERENCE_DIR). Builds the reduced backbone of tests/e2e_model.py
from transformers' Qwen3.5 decoder layers (the modules the reference's HF stack
runs, d3trt/model/hf_stack.py:15-40), with every Linear of the layers replaced by
the reference's W8A8 FP8 QuantLinear (d3trt/model/quant.py:103-197, emulated on
the CPU), all in bf16. Then runs the reference's state-once schedule exactly as
HFStack does (hf_stack.py:44-66: embeddings, M-RoPE positions, D3Core.state and
D3Core.questions with recurrent_max_tokens=0) and its readout (hf_stack.py:67-84,
fp32 logits and softmax). Records the per-block probabilities (zero past each
block's count) and the final-norm hidden rows. The fixture is committed; this
script is only needed to regenerate it.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(OUT.parent))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("D3_REFERENCE_DIR"))
    args = ap.parse_args()
    if not args.reference or not Path(args.reference, "d3trt").is_dir():
        raise SystemExit("pass --reference <d3-turbo-trt checkout> (or set D3_REFERENCE_DIR)")
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from d3trt.model.core import D3Core  # noqa: E402
    from d3trt.model.quant import QuantLinear  # noqa: E402
    from transformers.models.qwen3_5 import modeling_qwen3_5 as m  # noqa: E402
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig  # noqa: E402

    import e2e_model as em

    torch.set_grad_enabled(False)
    torch.manual_seed(0)
    c = em.CONFIG
    cfg = Qwen3_5TextConfig(
        vocab_size=em.VOCAB, hidden_size=c["hidden_size"], intermediate_size=c["intermediate_size"],
        num_hidden_layers=len(c["layer_types"]), num_attention_heads=c["num_attention_heads"],
        num_key_value_heads=c["num_key_value_heads"], head_dim=c["head_dim"],
        linear_num_key_heads=c["linear_num_key_heads"], linear_num_value_heads=c["linear_num_value_heads"],
        linear_key_head_dim=c["linear_key_head_dim"], linear_value_head_dim=c["linear_value_head_dim"],
        linear_conv_kernel_dim=c["linear_conv_kernel_dim"], rms_norm_eps=c["rms_norm_eps"],
        layer_types=c["layer_types"],
        rope_parameters={"rope_type": "default", "rope_theta": c["rope_theta"],
                         "partial_rotary_factor": c["partial_rotary_factor"], "mrope_section": [11, 11, 10],
                         "mrope_interleaved": True},
    )
    cfg._attn_implementation = "sdpa"
    layers = torch.nn.ModuleList([m.Qwen3_5DecoderLayer(cfg, i) for i in range(len(c["layer_types"]))])
    final_norm = m.Qwen3_5RMSNorm(c["hidden_size"], eps=c["rms_norm_eps"])
    embed = torch.nn.Embedding(em.VOCAB, c["hidden_size"])
    rotary = m.Qwen3_5TextRotaryEmbedding(cfg)
    weights = em.make_weights()
    holder = torch.nn.Module()
    holder.layers, holder.norm, holder.embed_tokens = layers, final_norm, embed
    holder.to(torch.bfloat16)
    missing, unexpected = holder.load_state_dict(weights, strict=False)
    assert not unexpected and not [k for k in missing if "rotary" not in k], (missing, unexpected)
    # every Linear of the layers -> the reference's FP8 QuantLinear (emulated on the CPU)
    for layer in layers:
        for parent in [mod for mod in layer.modules()]:
            for name, child in list(parent.named_children()):
                if isinstance(child, torch.nn.Linear):
                    ql = QuantLinear(child.in_features, child.out_features, mode="fp8", dtype=torch.bfloat16,
                                     device="cpu")
                    ql.load_full(child.weight.data)
                    setattr(parent, name, ql)
    core = D3Core(layers=layers, layer_types=c["layer_types"], final_norm=final_norm, rotary_emb=rotary,
                  apply_rotary=m.apply_rotary_pos_emb, attention_state="sdpa", attention_question="sdpa",
                  recurrent_max_tokens=0)

    state_ids, ids, lengths, counts, readout = em.make_request()
    embeds = embed(state_ids)
    positions = torch.arange(state_ids.shape[1]).view(1, 1, -1).expand(3, 1, -1)
    snapshot = core.state(embeds, rotary(embeds, positions))
    q_embeds = embed(ids)
    steps = (state_ids.shape[1] + torch.arange(ids.shape[1])).view(1, 1, -1)
    hidden = core.questions(snapshot, q_embeds, lengths, rotary(q_embeds, steps.expand(3, ids.shape[0], -1)))
    logits = hidden.float() @ readout.T
    counts_t = torch.as_tensor(counts)[:, None]
    logits = logits.masked_fill(torch.arange(em.OPTIONS)[None] >= counts_t, float("-inf"))
    probs = logits.softmax(-1)
    assert core.stats.attention_question == "sdpa" and core.stats.delta.startswith("torch-chunk")
    np.savez_compressed(OUT / "e2e_4layer.npz", probs=probs.numpy().astype(np.float32),
                        hidden=hidden.float().numpy(), counts=np.array(counts, np.int32),
                        lengths=np.array(lengths, np.int32))
    print("e2e_4layer.npz", (OUT / "e2e_4layer.npz").stat().st_size, "max p", float(probs.max()))


if __name__ == "__main__":
    main()
