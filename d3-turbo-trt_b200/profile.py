"""Run one hot-path kernel on one configuration a fixed number of times.

    python -m d3_turbo_trt_b200.profile --kernel attention --config cfg3a --launches 3

Meant as the target of an ``ncu`` capture (one kernel, a few launches, a small
device footprint) and as a quick device-time probe: it prints the median
CUDA-event time per launch and the algorithmic work per launch. Configs follow
cfg3a (4096-token state + 16 x 64-token blocks), cfg3b (16384 +
255 x 48), cfg5 (16384 + 255 x 64 on one GPU: the CTA-pair attention kernel),
model_d256 (cfg3a's blocks and state at 24/4 heads, head_dim 256: the D = 256
kernel's split launch), state4k (the state pass of cfg3a), cfg2 (W8A8 4096 x 5120 x 13824),
cfg4 (readout 255 x 5120 x 255; snapshot: the 64-layer state snapshot at a
4096-token state, packed by one copy launch; gdn: one GDN layer's question pass,
255 blocks x 48 tokens x 48 value heads; gdn_state: one GDN layer's state pass,
4096 tokens x 48 value heads with a final state; gated_norm_fp8, causal_conv,
qk_norm_rope: the backbone's glue kernels at the question pass's 255 x 48 tokens).
Inputs are seeded synthetic tensors.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch

from .kernels import prefix_bidir as pb
from .model import quant
from .model import gdn
from .model.readout import probabilities_tensor
from .model.snapshot import AttentionEntry, DeltaEntry, SnapshotArena, SnapshotLayout, copy_segments

ATTN = {
    "cfg3a": dict(B=16, H=32, Hkv=4, L=64, D=128, S=4096),
    "cfg3b": dict(B=255, H=32, Hkv=4, L=48, D=128, S=16384),
    "cfg1": dict(B=8, H=8, Hkv=2, L=32, D=64, S=512),
    "cfg5": dict(B=255, H=32, Hkv=4, L=64, D=128, S=16384),
    # config 3a's blocks and state at the model's own attention shape (head_dim 256)
    "model_d256": dict(B=16, H=24, Hkv=4, L=64, D=256, S=4096),
}


def _attention(cfg: str, dev: torch.device):
    c = ATTN[cfg]
    g = torch.Generator().manual_seed(0)
    B, H, Hkv, L, D, S = (c[k] for k in ("B", "H", "Hkv", "L", "D", "S"))
    q = torch.randn(B, L, H, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    kq = torch.randn(B, L, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    vq = torch.randn(B, L, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    ks = torch.randn(S, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(1, 0, 2)
    vs = torch.randn(S, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(1, 0, 2)
    out = torch.empty(B, H, L, D, dtype=torch.bfloat16, device=dev)
    lens = [L] * B
    flops = 4.0 * H * D * B * L * (S + L)
    return (lambda: pb.prefix_bidir_attention(q, ks, vs, kq, vq, lens, scale=D ** -0.5, out=out)), {"flops": flops}


def _state(dev: torch.device, tokens: int = 4096):
    g = torch.Generator().manual_seed(1)
    H, Hkv, D = 32, 4, 128
    q = torch.randn(1, tokens, H, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    k = torch.randn(1, tokens, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    v = torch.randn(1, tokens, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    return (lambda: pb.state_attention(q, k, v, scale=D ** -0.5)), {"flops": 4.0 * H * D * tokens * tokens}


def _gemm(mode: str, dev: torch.device, M=4096, K=5120, N=13824):
    g = torch.Generator().manual_seed(2)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    layer = quant.QuantLinear(K, N, mode=mode, dtype=torch.bfloat16, device=dev)
    layer.load_full(w)
    qa, sa = quant.quantize_rows(x, mode)
    fn = lambda: quant.scaled_mm(qa, layer.weight, sa, layer.weight_scale, out_dtype=torch.bfloat16)
    return fn, {"flops": 2.0 * M * N * K, "bytes": M * K + N * K + M * N * 2}


def _act_quant(mode: str, dev: torch.device, M=4096, K=5120):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    return (lambda: quant.quantize_rows(x, mode)), {"bytes": M * K * 3 + M * 4}


def _readout(dev: torch.device, B=255, K=5120, n_opt=255):
    g = torch.Generator().manual_seed(4)
    h = torch.randn(B, K, generator=g).to(torch.bfloat16).to(dev)
    r = (torch.randn(n_opt, K, generator=g) * 0.02).to(dev)
    counts = torch.full((B,), n_opt, dtype=torch.int32, device=dev)
    return (lambda: probabilities_tensor(h, r, counts, temperature=1.0)), {
        "flops": 2.0 * B * K * n_opt, "bytes": B * K * 2 + n_opt * K * 4 + B * n_opt * 4}


def state_snapshot(dev: torch.device, S: int = 4096, layers: int = 64, Hkv: int = 4, D: int = 128,
                   conv_dim: int = 10240, Hv: int = 48, dk: int = 128, dv: int = 128, window: int = 3,
                   shared_parent: bool = False) -> list:
    """The snapshot D3Core's state pass leaves for the 64-layer model (every 4th layer full
    attention): K token-major after RoPE and V as a transposed view of v_proj's output
    (core.py:233-251); the GDN conv tail as the last ``window`` columns of the whole
    in_proj_qkv output and an fp32 recurrent state (core.py:301-358). ``shared_parent``
    cuts every tail from one in_proj_qkv buffer instead of one per layer (same copy work,
    80 MiB instead of 3.75 GiB on the device)."""
    g = torch.Generator(device=dev).manual_seed(5)
    snap, mixed = [], None
    for i in range(layers):
        if i % 4 == 3:
            k = torch.randn(1, S, Hkv, D, generator=g, device=dev).to(torch.bfloat16).transpose(1, 2)
            v = torch.randn(1, S, Hkv * D, generator=g, device=dev).to(torch.bfloat16)
            snap.append(AttentionEntry(keys=k, values=v.view(1, S, Hkv, D).transpose(1, 2)))
        else:
            if mixed is None or not shared_parent:
                mixed = torch.randn(1, S, conv_dim, generator=g, device=dev).to(torch.bfloat16).transpose(1, 2)
            rec = torch.randn(1, Hv, dk, dv, generator=g, device=dev)
            snap.append(DeltaEntry(tail=mixed[:, :, -window:], recurrent=rec))
    return snap


def _snapshot(dev: torch.device):
    snap = state_snapshot(dev, shared_parent=True)
    layout = SnapshotLayout.of(snap)
    arena = SnapshotArena(layout.nbytes, dev)
    block = arena.allocate(layout.nbytes)
    table = layout.table(snap, arena.buffer.data_ptr() + block.offset)

    def run():  # holds the snapshot, arena and block alive with the table
        copy_segments(table, dev)
        return snap, arena, block

    return run, {"bytes": 2 * layout.tensor_bytes}


def gdn_question_inputs(dev: torch.device, B: int = 255, T: int = 48, H: int = 16, HV: int = 48, K: int = 128,
                        V: int = 128, seed: int = 6) -> dict:
    """One GDN layer's question pass as D3Core runs it at BASELINE config 3b/4 (255 blocks of 48
    tokens; 16 q/k heads, 48 value heads of 128, core.py:333-347), state from the snapshot."""
    g = torch.Generator(device=dev).manual_seed(seed)
    return {
        "q": torch.randn(B, T, H, K, generator=g, device=dev).to(torch.bfloat16),
        "k": torch.randn(B, T, H, K, generator=g, device=dev).to(torch.bfloat16),
        "v": torch.randn(B, T, HV, V, generator=g, device=dev).to(torch.bfloat16),
        "g": -torch.rand(B, T, HV, generator=g, device=dev) * 0.5,
        "beta": torch.sigmoid(torch.randn(B, T, HV, generator=g, device=dev)).to(torch.bfloat16),
        "h0": torch.randn(1, HV, K, V, generator=g, device=dev) * 0.5,
    }


def _gdn(dev: torch.device, algo: str):
    x = gdn_question_inputs(dev)
    B = x["q"].shape[0]
    out = torch.empty_like(x["v"])
    fn = lambda: gdn.gated_delta_rule(x["q"], x["k"], x["v"], g=x["g"], beta=x["beta"],
                                      initial_state=x["h0"].expand(B, -1, -1, -1), out=out, algo=algo)
    B, T, H, K = x["q"].shape
    HV, V = x["v"].shape[2:]
    # chunked form: K K^T, K S0, Q K^T, Q S0 and P V' on two 64-token blocks per 128-row tile
    flops = 2.0 * 5 * 128 * 128 * 128 * ((B + 1) // 2) * HV if algo == "chunk" else 2.0 * 3 * B * T * HV * K * V
    return fn, {"flops": flops}


def _gdn_state(dev: torch.device, T: int = 4096, H: int = 16, HV: int = 48, K: int = 128, V: int = 128):
    """One GDN layer's state pass (config 4): one row of 4096 tokens, final state, the inter-chunk form."""
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(1, T, H, K, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, T, H, K, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(1, T, HV, V, generator=g, device=dev).to(torch.bfloat16)
    gl = -torch.rand(1, T, HV, generator=g, device=dev) * 0.5
    beta = torch.sigmoid(torch.randn(1, T, HV, generator=g, device=dev)).to(torch.bfloat16)
    fn = lambda: gdn.chunk_gated_delta_rule(q, k, v, g=gl, beta=beta, initial_state=None, output_final_state=True)
    # tensor products per (64-token chunk, value head): K K^T, Q K^T, W, U (64 x 64 x 128 each),
    # [W; Q] S (2 x 64 x 128 x 128), K^T V'' (128 x 64 x 128), P V' (64 x 64 x 128)
    macs = 4 * 64 * 64 * 128 + 2 * 64 * 128 * 128 + 128 * 64 * 128 + 64 * 64 * 128
    return fn, {"flops": 2.0 * macs * ((T + 63) // 64) * HV}


def _glue(kernel: str, dev: torch.device, rows: int = 255, T: int = 48):
    """config 4's question pass (255 blocks x 48 tokens): the GDN output's gated norm + quant
    (48 heads x 128), the GDN causal conv + SiLU (conv_dim 10240, a 3-token tail), or the
    attention queries' norm + partial rotary (32 heads x 128, the q half of q_proj's output)."""
    from .model import fused
    from .model.backbone import BackboneConfig, rotary_tables
    from .model.conv import causal_conv1d_silu

    g = torch.Generator(device=dev).manual_seed(6)
    M = rows * T
    if kernel == "gated_norm_fp8":
        x = (torch.randn(M, 6144, generator=g, device=dev) * 0.3).to(torch.bfloat16)
        z = torch.randn(M, 6144, generator=g, device=dev).to(torch.bfloat16)
        w = (1 + torch.randn(128, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        return (lambda: fused.gated_rmsnorm_quant(x, z, w, 1e-6, 128, "fp8")), {"bytes": M * 6144 * 5 + M * 4}
    if kernel == "causal_conv":
        x = torch.randn(rows, T, 10240, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(10240, 1, 4, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        tail = torch.randn(rows, 10240, 3, generator=g, device=dev).to(torch.bfloat16)
        return (lambda: causal_conv1d_silu(x, w, tail)), {"bytes": 2 * x.numel() * 2}
    qg = torch.randn(rows, T, 32, 256, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(128, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    positions = (torch.arange(T, device=dev)[None] + 4096).expand(rows, T)
    cos, sin = rotary_tables(BackboneConfig(), positions, torch.bfloat16)
    return (lambda: fused.qk_norm_rope(qg[..., :128], w, cos, sin, 1e-6)), {"bytes": M * 32 * 128 * 4}


def build(kernel: str, config: str, dev: torch.device):
    if kernel in ("gated_norm_fp8", "causal_conv", "qk_norm_rope"):
        return _glue(kernel, dev)
    if kernel == "attention":
        return _state(dev) if config == "state4k" else _attention(config, dev)
    if kernel == "gemm_fp8":
        return _gemm("fp8", dev)
    if kernel == "gemm_int8":
        return _gemm("int8", dev)
    if kernel == "act_quant_fp8":
        return _act_quant("fp8", dev)
    if kernel == "act_quant_int8":
        return _act_quant("int8", dev)
    if kernel == "readout":
        return _readout(dev)
    if kernel == "snapshot":
        return _snapshot(dev)
    if kernel == "gdn":
        return _gdn(dev, "chunk")
    if kernel == "gdn_recurrent":
        return _gdn(dev, "recurrent")
    if kernel == "gdn_state":
        return _gdn_state(dev)
    raise SystemExit(f"unknown kernel {kernel!r}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True,
                    choices=["attention", "gemm_fp8", "gemm_int8", "act_quant_fp8", "act_quant_int8", "readout",
                             "snapshot", "gdn", "gdn_recurrent", "gdn_state", "gated_norm_fp8", "causal_conv",
                             "qk_norm_rope"])
    ap.add_argument("--config", default="cfg3a", choices=[*ATTN, "state4k", "cfg2", "cfg4"])
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fn, work = build(args.kernel, args.config, dev)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.launches):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(1_000_000)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    rep = {"kernel": args.kernel, "config": args.config, "ms": ms}
    if "flops" in work:
        rep["tflops"] = work["flops"] / ms / 1e9
    if "bytes" in work:
        rep["gbs"] = work["bytes"] / ms / 1e6
    print(json.dumps(rep))


if __name__ == "__main__":
    main()
