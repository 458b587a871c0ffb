"""A reduced, seeded d3 backbone for the end-to-end parity check (test infrastructure).

The weights and inputs are generated on the CPU from fixed seeds, so the fixture
script (tests/golden/make_e2e_golden.py, which runs the reference's own D3Core
on transformers' Qwen3.5 layers) and the GPU test (which runs
d3_turbo_trt_b200.model.backbone.D3Backbone) see the same model and the same
request. The residual branches' output projections are scaled by BRANCH (see
there). The shape keeps the model's structure at a size the CPU runs in
seconds: 3 Gated DeltaNet layers and 1 full-attention layer (the model's 3:1
pattern), head_dim 128 for both mixers, the real model's ratios of heads
(GQA 4 for attention, 2 value heads per key head in the GDN layers), every
projection quantizable, a 255-way readout.
"""

from __future__ import annotations

import torch

CONFIG = dict(
    hidden_size=1024,
    intermediate_size=2048,
    num_attention_heads=8,
    num_key_value_heads=2,
    head_dim=128,
    linear_num_key_heads=8,
    linear_num_value_heads=16,
    linear_key_head_dim=128,
    linear_value_head_dim=128,
    linear_conv_kernel_dim=4,
    rms_norm_eps=1e-6,
    rope_theta=10_000_000.0,
    partial_rotary_factor=0.25,
    layer_types=["linear_attention", "linear_attention", "linear_attention", "full_attention"],
)
VOCAB = 4096
STATE_TOKENS = 512
BLOCKS = 12
BLOCK_TOKENS = 48
OPTIONS = 255
WEIGHT_SEED = 2024
INPUT_SEED = 7
READOUT_SEED = 139
# Scale of the residual branches' output projections (o_proj, out_proj, down_proj).
# As in trained models, each layer adds a small update to a larger residual stream.
# With unit-scale branches a random 4-layer stack is chaotic under W8A8 FP8: the
# activation codes' 3-bit mantissa turns a relative difference d between two valid
# implementations into ~0.25*sqrt(d) per quantised projection, and the reference's
# own two paths (fp32 vs bf16 L2 norm of q/k in the GDN scan) then differ by 0.035
# in probability. At 0.1 they differ by well under the 1e-2 gate.
BRANCH = 0.1


def make_weights(config: dict = CONFIG, seed: int = WEIGHT_SEED) -> dict[str, torch.Tensor]:
    """Every parameter by the model's own name, bf16, from one CPU generator (fixed order)."""
    g = torch.Generator().manual_seed(seed)
    c = config
    H, I = c["hidden_size"], c["intermediate_size"]
    D, Hq, Hkv = c["head_dim"], c["num_attention_heads"], c["num_key_value_heads"]
    HK, HV = c["linear_num_key_heads"], c["linear_num_value_heads"]
    Dk, Dv = c["linear_key_head_dim"], c["linear_value_head_dim"]
    conv_dim = 2 * HK * Dk + HV * Dv

    def normal(*shape, std):
        return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)

    w: dict[str, torch.Tensor] = {"embed_tokens.weight": normal(VOCAB, H, std=1.0),
                                  "norm.weight": normal(H, std=0.1)}
    for i, kind in enumerate(c["layer_types"]):
        p = f"layers.{i}."
        w[p + "input_layernorm.weight"] = normal(H, std=0.1)
        w[p + "post_attention_layernorm.weight"] = normal(H, std=0.1)
        if kind == "full_attention":
            a = p + "self_attn."
            w[a + "q_proj.weight"] = normal(2 * Hq * D, H, std=H ** -0.5)
            w[a + "k_proj.weight"] = normal(Hkv * D, H, std=H ** -0.5)
            w[a + "v_proj.weight"] = normal(Hkv * D, H, std=H ** -0.5)
            w[a + "o_proj.weight"] = normal(H, Hq * D, std=BRANCH * (Hq * D) ** -0.5)
            w[a + "q_norm.weight"] = normal(D, std=0.1)
            w[a + "k_norm.weight"] = normal(D, std=0.1)
        else:
            a = p + "linear_attn."
            w[a + "in_proj_qkv.weight"] = normal(conv_dim, H, std=H ** -0.5)
            w[a + "in_proj_z.weight"] = normal(HV * Dv, H, std=H ** -0.5)
            w[a + "in_proj_b.weight"] = normal(HV, H, std=H ** -0.5)
            w[a + "in_proj_a.weight"] = normal(HV, H, std=H ** -0.5)
            w[a + "conv1d.weight"] = normal(conv_dim, 1, c["linear_conv_kernel_dim"], std=0.5)
            w[a + "dt_bias"] = torch.ones(HV, dtype=torch.bfloat16)
            A = torch.empty(HV).uniform_(0.05, 2.0, generator=g)
            w[a + "A_log"] = torch.log(A).to(torch.bfloat16)
            w[a + "norm.weight"] = (1.0 + torch.randn(Dv, generator=g) * 0.1).to(torch.bfloat16)
            w[a + "out_proj.weight"] = normal(H, HV * Dv, std=BRANCH * (HV * Dv) ** -0.5)
        w[p + "mlp.gate_proj.weight"] = normal(I, H, std=H ** -0.5)
        w[p + "mlp.up_proj.weight"] = normal(I, H, std=H ** -0.5)
        w[p + "mlp.down_proj.weight"] = normal(H, I, std=BRANCH * I ** -0.5)
    return w


def make_request(config: dict = CONFIG, seed: int = INPUT_SEED):
    """(state ids [1, S], question ids [B, W] right-padded with 0, lengths, counts, readout [255, H] fp32)."""
    g = torch.Generator().manual_seed(seed)
    state = torch.randint(0, VOCAB, (1, STATE_TOKENS), generator=g)
    lengths = torch.randint(1, BLOCK_TOKENS + 1, (BLOCKS,), generator=g).tolist()
    lengths[0] = BLOCK_TOKENS
    lengths[1] = 1
    ids = torch.zeros(BLOCKS, BLOCK_TOKENS, dtype=torch.long)
    for r, n in enumerate(lengths):
        ids[r, :n] = torch.randint(0, VOCAB, (n,), generator=g)
    counts = torch.randint(2, OPTIONS + 1, (BLOCKS,), generator=g).tolist()
    counts[0] = OPTIONS
    # N(0, 0.02) at the model's 5120 wide hidden state; scaled so logits keep that spread here.
    # Its seed gives every block a top-1 logit margin >= 0.3 under the reference: argmax
    # agreement is only a well-posed check where the top answer is not a near tie.
    gr = torch.Generator().manual_seed(READOUT_SEED)
    readout = torch.randn(OPTIONS, config["hidden_size"], generator=gr) * (0.02 * (5120 / config["hidden_size"]) ** 0.5)
    return state, ids, lengths, counts, readout
