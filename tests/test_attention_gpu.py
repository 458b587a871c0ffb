"""GPU parity of the prefix-bidirectional attention against the oracle
(ops.sdpa_questions / sdpa_state restated) and the golden vectors recorded from
the reference: within 2e-2 max-abs (the BASELINE tolerance), and in practice
near bf16 output rounding."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import attention as oattn

from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.kernels import prefix_bidir as pb
from d3_turbo_trt_b200.model import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


def _rand(shape, g, dtype=torch.bfloat16):
    return torch.randn(*shape, generator=g).to(dtype)


def test_cfg1_golden_strided_views():
    """BASELINE config 1 ([768, 8, 64] over a 512-token state + 8 x 32), read
    through strided views of the token-major sequence: no copies."""
    g = load_golden("attn_cfg1.npz")
    state, nb, lq, heads, kv_heads, dim = (int(v) for v in g["meta"])
    scale = float(g["scale"])
    Q = bf16_from_bits(g["Q"]).to(DEV)
    K = bf16_from_bits(g["K"]).to(DEV)
    V = bf16_from_bits(g["V"]).to(DEV)
    ks, vs = K[:state].transpose(0, 1), V[:state].transpose(0, 1)  # [Hkv, S, D], token-major
    qq = Q[state:].view(nb, lq, heads, dim).permute(0, 2, 1, 3)
    kq = K[state:].view(nb, lq, kv_heads, dim).permute(0, 2, 1, 3)
    vq = V[state:].view(nb, lq, kv_heads, dim).permute(0, 2, 1, 3)
    out_q, kernel = ops.question_attention(qq, ks, vs, kq, vq, [lq] * nb, scale=scale, return_kernel=True)
    assert kernel == "sm100a"
    out_s = ops.flash_state(Q[:state].transpose(0, 1)[None], ks[None], vs[None], scale=scale)
    out = torch.cat([out_s[0].transpose(0, 1), out_q.permute(0, 2, 1, 3).reshape(nb * lq, heads, dim)], 0)
    err = np.abs(out.float().cpu().numpy() - g["out"]).max()
    assert err <= TOL, err
    assert _lib.device_error() == 0


@pytest.mark.parametrize("case", ["d32_g2", "d64_g3", "d256_g1", "d128_g8"])
def test_ragged_golden(case):
    g = load_golden("attn_ragged.npz")
    t = {k: bf16_from_bits(g[f"{case}_{k}"]).to(DEV) for k in ("q", "ks", "vs", "kq", "vq")}
    lens = g[f"{case}_lens"].tolist()
    out = pb.prefix_bidir_attention(t["q"], t["ks"], t["vs"], t["kq"], t["vq"], lens, scale=float(g[f"{case}_scale"]))
    got = out.float().cpu().numpy()
    ref = g[f"{case}_out"]
    assert np.abs(got - ref).max() <= TOL
    for b, n in enumerate(lens):
        assert np.all(got[b, :, n:] == 0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cfg3a_shape_against_oracle(dtype):
    """BASELINE config 3a shapes: 4096-token state + 16 blocks x 64, H32/Hkv4/D128;
    the oracle checks every block (two ragged)."""
    g = torch.Generator().manual_seed(11)
    B, H, Hkv, L, D, S = 16, 32, 4, 64, 128, 4096
    q = _rand((B, L, H, D), g, dtype).permute(0, 2, 1, 3)  # model layout: [B, L, H, D] memory
    ks = _rand((S, Hkv, D), g, dtype).permute(1, 0, 2)      # token-major state
    vs = _rand((S, Hkv, D), g, dtype).permute(1, 0, 2)
    kq = _rand((B, L, Hkv, D), g, dtype).permute(0, 2, 1, 3)
    vq = _rand((B, L, Hkv, D), g, dtype).permute(0, 2, 1, 3)
    lens = [64] * B
    lens[5] = 37
    lens[9] = 1
    out = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens, scale=D**-0.5)
    got = out.float().cpu()
    ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
    err = (got - ref).abs().amax(dim=(1, 2, 3))
    assert float(err.max()) <= TOL, err
    assert torch.all(got[5, :, 37:] == 0) and torch.all(got[9, :, 1:] == 0)


def test_head_major_state_and_empty_blocks():
    g = torch.Generator().manual_seed(12)
    B, H, Hkv, L, D, S = 4, 16, 2, 48, 128, 300
    q = _rand((B, H, L, D), g)
    ks, vs = _rand((Hkv, S, D), g), _rand((Hkv, S, D), g)  # head-major contiguous
    kq, vq = _rand((B, Hkv, L, D), g), _rand((B, Hkv, L, D), g)
    lens = [48, 0, 17, 48]
    out = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens, scale=0.09)
    ref = oattn.questions(q, ks, vs, kq, vq, lens, 0.09, dtype=torch.float32)
    assert float((out.float().cpu() - ref).abs().max()) <= TOL
    assert torch.all(out[1] == 0)
    z = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), [0] * B, scale=0.09)
    assert torch.all(z == 0)


@pytest.mark.parametrize("tokens,heads,kv_heads,dim", [(1000, 16, 2, 128), (257, 8, 8, 64), (130, 4, 1, 256)])
def test_state_pass_against_oracle(tokens, heads, kv_heads, dim):
    g = torch.Generator().manual_seed(13)
    q = _rand((1, heads, tokens, dim), g)
    k = _rand((1, kv_heads, tokens, dim), g)
    v = _rand((1, kv_heads, tokens, dim), g)
    out = ops.flash_state(q.to(DEV), k.to(DEV), v.to(DEV), scale=dim**-0.5)
    ref = oattn.state(q, k, v, dim**-0.5, dtype=torch.float32)
    assert float((out.float().cpu() - ref).abs().max()) <= TOL


def test_large_logits_stay_finite():
    """Scores far from zero exercise the lazy rescale (max jumps by > 2^8)."""
    g = torch.Generator().manual_seed(14)
    B, H, Hkv, L, D, S = 2, 8, 1, 32, 64, 512
    q = _rand((B, H, L, D), g) * 4
    ks = _rand((Hkv, S, D), g) * 4
    ks[:, 300:] *= 3  # later keys dominate: the running max grows mid-stream
    vs = _rand((Hkv, S, D), g)
    kq, vq = _rand((B, Hkv, L, D), g) * 4, _rand((B, Hkv, L, D), g)
    out = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), [32, 20], scale=0.5)
    ref = oattn.questions(q, ks, vs, kq, vq, [32, 20], 0.5, dtype=torch.float64)
    got = out.float().cpu()
    assert torch.isfinite(got).all()
    assert float((got - ref).abs().max()) <= TOL


def test_preallocated_strided_output_and_tensor_lengths():
    g = torch.Generator().manual_seed(15)
    B, H, Hkv, L, D, S = 3, 8, 2, 16, 64, 128
    q = _rand((B, H, L, D), g).to(DEV)
    ks, vs = _rand((Hkv, S, D), g).to(DEV), _rand((Hkv, S, D), g).to(DEV)
    kq, vq = _rand((B, Hkv, L, D), g).to(DEV), _rand((B, Hkv, L, D), g).to(DEV)
    lens = torch.tensor([16, 3, 9], dtype=torch.int32, device=DEV)
    buf = torch.full((B, L, H, D), 7.0, dtype=torch.bfloat16, device=DEV)
    out = buf.permute(0, 2, 1, 3)
    pb.prefix_bidir_attention(q, ks, vs, kq, vq, lens, scale=0.125, out=out)
    ref = oattn.questions(q.cpu(), ks.cpu(), vs.cpu(), kq.cpu(), vq.cpu(), [16, 3, 9], 0.125, dtype=torch.float32)
    assert float((out.float().cpu() - ref).abs().max()) <= TOL


def _long_state_case(seed, B, L, S=16384, H=32, Hkv=4, D=128):
    g = torch.Generator().manual_seed(seed)
    q = _rand((B, L, H, D), g).permute(0, 2, 1, 3)
    ks = _rand((S, Hkv, D), g).permute(1, 0, 2)
    vs = _rand((S, Hkv, D), g).permute(1, 0, 2)
    kq = _rand((B, L, Hkv, D), g).permute(0, 2, 1, 3)
    vq = _rand((B, L, Hkv, D), g).permute(0, 2, 1, 3)
    return q, ks, vs, kq, vq


@pytest.mark.parametrize("name,B,L", [("cfg3b", 255, 48), ("cfg5", 255, 64)])
def test_long_state_against_oracle(name, B, L):
    """BASELINE configs 3b and 5: a 16384-token state and 255 question blocks
    (48 or 64 tokens), H32/Hkv4/D128. Ten blocks are checked against the oracle:
    the first, the last, three ragged ones and five spread over the batch."""
    q, ks, vs, kq, vq = _long_state_case(21 if name == "cfg3b" else 22, B, L)
    lens = [L] * B
    lens[3], lens[130], lens[B - 2] = L - 1, 1, L // 2 + 3
    out = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens, scale=128**-0.5)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    for b in (0, 3, 41, 97, 130, 166, 201, 229, B - 2, B - 1):
        ref = oattn.questions(q[b : b + 1], ks, vs, kq[b : b + 1], vq[b : b + 1], [lens[b]], 128**-0.5,
                              dtype=torch.float32)
        got = out[b : b + 1].float().cpu()
        assert float((got - ref).abs().max()) <= TOL, b
        assert torch.all(got[0, :, lens[b]:] == 0)


def test_head_dim_256_at_4k_state():
    """The model's own attention shape (24 query heads, 4 KV heads, head_dim 256:
    a GQA group of 6, which does not divide the 128-row tile) over a 4096-token
    state, question pass and state pass, against the oracle."""
    g = torch.Generator().manual_seed(23)
    B, H, Hkv, L, D, S = 6, 24, 4, 48, 256, 4096
    q = _rand((B, L, H, D), g).permute(0, 2, 1, 3)
    ks = _rand((S, Hkv, D), g).permute(1, 0, 2)
    vs = _rand((S, Hkv, D), g).permute(1, 0, 2)
    kq = _rand((B, L, Hkv, D), g).permute(0, 2, 1, 3)
    vq = _rand((B, L, Hkv, D), g).permute(0, 2, 1, 3)
    lens = [48, 13, 48, 1, 47, 48]
    out = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens, scale=D**-0.5)
    ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
    assert float((out.float().cpu() - ref).abs().max()) <= TOL
    # state pass over the same 4096 tokens (S = 0 in the kernel): rows spread over the state
    qs = _rand((1, S, H, D), g).permute(0, 2, 1, 3)
    st = ops.flash_state(qs.to(DEV), ks[None].to(DEV), vs[None].to(DEV), scale=D**-0.5)
    rows = torch.tensor([0, 1, 127, 128, 2049, 4094, 4095])
    ref_s = oattn.state(qs[:, :, rows], ks[None], vs[None], D**-0.5, dtype=torch.float32)
    assert float((st[:, :, rows.to(DEV)].float().cpu() - ref_s).abs().max()) <= TOL
    assert _lib.device_error() == 0


def test_d256_single_issuer_kernel_in_a_subprocess():
    """head_dim 256 runs on the two-issuer kernel; D3B_ATTN_D256=single (read
    once per process) selects the one-issuer kernel. Both, in a fresh process
    each, against the oracle on a ragged split launch and a whole-unit one."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys, torch\n"
        f"sys.path[:0] = [{str(root)!r}, {str(root / 'tests')!r}]\n"
        "import conftest\n"
        "from oracle import attention as oattn\n"
        "from d3_turbo_trt_b200 import _lib\n"
        "from d3_turbo_trt_b200.kernels import prefix_bidir as pb\n"
        "worst = 0.0\n"
        "for B, H, Hkv, S, L, lens in ((16, 24, 4, 4096, 64, None), (5, 20, 2, 300, 50, [50, 1, 0, 33, 49])):\n"
        "    g = torch.Generator().manual_seed(B)\n"
        "    q = torch.randn(B, L, H, 256, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)\n"
        "    ks = torch.randn(S, Hkv, 256, generator=g).to(torch.bfloat16).permute(1, 0, 2)\n"
        "    vs = torch.randn(S, Hkv, 256, generator=g).to(torch.bfloat16).permute(1, 0, 2)\n"
        "    kq = torch.randn(B, L, Hkv, 256, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)\n"
        "    vq = torch.randn(B, L, Hkv, 256, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)\n"
        "    lens = lens or [L] * B\n"
        "    out = pb.prefix_bidir_attention(*(t.cuda() for t in (q, ks, vs, kq, vq)), lens, scale=256 ** -0.5)\n"
        "    torch.cuda.synchronize()\n"
        "    assert _lib.device_error() == 0\n"
        "    ref = oattn.questions(q, ks, vs, kq, vq, lens, 256 ** -0.5, dtype=torch.float32)\n"
        "    worst = max(worst, float((out.float().cpu() - ref).abs().max()))\n"
        "print(worst)\n"
    )
    for mode in ("single", "dual"):
        env = dict(os.environ, D3B_ATTN_D256=mode)
        res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
        assert res.returncode == 0, res.stderr[-2000:]
        assert float(res.stdout.strip().splitlines()[-1]) <= TOL, mode


def test_split_d256_pieces_without_real_keys():
    """A D = 256 split launch (64-key tiles) whose tail units hold a few real
    tokens of a long block: their last piece starts past the block's last real
    key tile and writes an empty partial (l = 0), the middle piece has a few
    key tiles. A first launch with full blocks leaves every partial slot
    filled, so a piece that did not write its slot would merge stale rows."""
    B, H, Hkv, S, L, D = 3, 2, 1, 64, 4096, 256
    assert int(_lib.lib().d3b_prefix_bidir_workspace_size(B, H, Hkv, S, L, D)) > 0
    g = torch.Generator().manual_seed(36)
    q = _rand((B, H, L, D), g)
    ks, vs = _rand((Hkv, S, D), g), _rand((Hkv, S, D), g)
    kq, vq = _rand((B, Hkv, L, D), g), _rand((B, Hkv, L, D), g)
    args = (q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV))
    pb.prefix_bidir_attention(*args, [L] * B, scale=D**-0.5)
    lens = [L, 1000, 1500]
    out = pb.prefix_bidir_attention(*args, lens, scale=D**-0.5)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
    got = out.float().cpu()
    assert float((got - ref).abs().max()) <= TOL
    for b, n in enumerate(lens):
        assert torch.all(got[b, :, n:] == 0)


@pytest.mark.parametrize("B,H,Hkv,S,L,D,seed", [(16, 24, 4, 1000, 64, 256, 41), (37, 24, 2, 500, 64, 128, 42),
                                                 (9, 24, 4, 300, 64, 64, 43), (5, 20, 2, 700, 50, 128, 44),
                                                 (4, 20, 2, 300, 50, 256, 45)])
def test_head_group_tiles_against_oracle(B, H, Hkv, S, L, D, seed):
    """GQA groups that do not divide the 128-row tile are split into head
    groups (G = 6 at 64 tokens: 3 tiles of 2 heads x 64 tokens; G = 12: 3
    groups of 4 heads x 32 tokens; G = 10 at 50 tokens: 4 tiles of 5 heads x 25
    tokens, 125 of 128 rows), each head group reading its KV head's keys: the
    D = 256 kernel, the D <= 128 kernel, ragged and empty blocks, against the
    oracle, and rows past each block's length zero."""
    g = torch.Generator().manual_seed(seed)
    q = _rand((B, L, H, D), g).permute(0, 2, 1, 3)
    ks, vs = _rand((S, Hkv, D), g).permute(1, 0, 2), _rand((S, Hkv, D), g).permute(1, 0, 2)
    kq, vq = _rand((B, L, Hkv, D), g).permute(0, 2, 1, 3), _rand((B, L, Hkv, D), g).permute(0, 2, 1, 3)
    lens = torch.randint(0, L + 1, (B,), generator=g).tolist()
    lens[0], lens[1], lens[-1] = L, 1, 0
    out = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens, scale=D**-0.5)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
    got = out.float().cpu()
    assert float((got - ref).abs().max()) <= TOL
    for b, n in enumerate(lens):
        assert torch.all(got[b, :, n:] == 0)


def test_device_lengths_out_of_range_are_reported():
    """A device lengths table is read by the kernel itself: values outside
    [0, L] are clamped (no access leaves the tensors) and reported through the
    device error word, which the caller reads with d3b_device_error; that
    launch's outputs are void, and the next launch after the word is cleared
    is exact again."""
    g = torch.Generator().manual_seed(24)
    B, H, Hkv, L, D, S = 4, 8, 2, 32, 128, 256
    q = _rand((B, H, L, D), g).to(DEV)
    ks, vs = _rand((Hkv, S, D), g).to(DEV), _rand((Hkv, S, D), g).to(DEV)
    kq, vq = _rand((B, Hkv, L, D), g).to(DEV), _rand((B, Hkv, L, D), g).to(DEV)
    assert _lib.device_error() == 0
    good = torch.tensor([32, 5, 0, 17], dtype=torch.int32, device=DEV)
    ref = pb.prefix_bidir_attention(q, ks, vs, kq, vq, good, scale=0.1)
    assert _lib.device_error() == 0
    bad = torch.tensor([1000, 5, -3, 17], dtype=torch.int32, device=DEV)
    pb.prefix_bidir_attention(q, ks, vs, kq, vq, bad, scale=0.1)
    # the launch's outputs are void (other CTAs stop early once the word is set); the word says why
    assert _lib.device_error() == pb.SITE_BAD_LENGTH
    assert _lib.device_error() == 0  # read-and-clear
    again = pb.prefix_bidir_attention(q, ks, vs, kq, vq, good, scale=0.1)
    assert torch.equal(again, ref) and _lib.device_error() == 0


@pytest.mark.parametrize("B,H,Hkv,S,L,D,seed", [(40, 8, 2, 8200, 300, 64, 25), (24, 32, 4, 8192, 64, 128, 27),
                                                 (21, 24, 4, 8192, 48, 128, 29), (16, 24, 4, 8192, 64, 128, 31),
                                                 (16, 24, 4, 4096, 64, 256, 35)])
def test_split_schedule_ragged_against_oracle(B, H, Hkv, S, L, D, seed):
    """Units of the last partial wave cut into pieces and merged through the
    workspace (long units, few waves): ragged and empty blocks, blocks longer
    than one key tile, head_dim 64, a GQA group of 6, and the D = 256 kernel at
    the model's own attention shape (24/4 heads). Also checked: the
    workspace's counters are zero again afterwards, a second launch gives the
    same bits, and the entry point without a workspace (one CTA per unit)
    agrees with the oracle too."""
    nbytes = int(_lib.lib().d3b_prefix_bidir_workspace_size(B, H, Hkv, S, L, D))
    assert nbytes > 0  # these shapes are split
    g = torch.Generator().manual_seed(seed)
    q = _rand((B, H, L, D), g)
    ks, vs = _rand((Hkv, S, D), g), _rand((Hkv, S, D), g)
    kq, vq = _rand((B, Hkv, L, D), g), _rand((B, Hkv, L, D), g)
    lens = torch.randint(0, L + 1, (B,), generator=g).tolist()
    lens[0], lens[-1] = L, 0
    args = (q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens)
    out = pb.prefix_bidir_attention(*args, scale=D**-0.5)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    ws = pb._WORKSPACES[(torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)]
    assert int(ws[:1024].count_nonzero()) == 0  # per-unit counts start the next launch at zero
    ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
    assert float((out.float().cpu() - ref).abs().max()) <= TOL
    out_again = pb.prefix_bidir_attention(*args, scale=D**-0.5)
    assert torch.equal(out, out_again)  # the merge order is fixed: same bits every launch
    out2 = torch.empty_like(out)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    st = _lib.lib().d3b_prefix_bidir(
        _lib.ptr(args[0]), _lib.i64_array(args[0].stride()[:3]), _lib.ptr(args[1]), _lib.ptr(args[2]),
        _lib.i64_array(args[1].stride()[:2]), _lib.ptr(args[3]), _lib.ptr(args[4]),
        _lib.i64_array(args[3].stride()[:3]), _lib.ptr(lens_d), B, H, Hkv, S, L, D, _lib.BF16, float(D**-0.5),
        _lib.ptr(out2), _lib.i64_array(out2.stride()[:3]), _lib.stream_of(out2))
    assert st == 0
    assert float((out2.float().cpu() - ref).abs().max()) <= TOL
    assert _lib.device_error() == 0


def test_workspace_shared_by_shapes():
    """One workspace serves every shape on a stream: a split shape with few
    split units followed by one with 104 (counts past the first shape's, where
    its partial slots would lie if the count region's size followed the shape)
    must both be exact, in both orders."""
    small, big = (24, 32, 4, 8192, 64, 128), (21, 24, 4, 8192, 48, 128)
    for seed, (B, H, Hkv, S, L, D) in ((31, small), (32, big), (33, small), (34, big)):
        assert int(_lib.lib().d3b_prefix_bidir_workspace_size(B, H, Hkv, S, L, D)) > 0
        g = torch.Generator().manual_seed(seed)
        q = _rand((B, H, L, D), g)
        ks, vs = _rand((Hkv, S, D), g), _rand((Hkv, S, D), g)
        kq, vq = _rand((B, Hkv, L, D), g), _rand((B, Hkv, L, D), g)
        lens = [L] * B
        out = pb.prefix_bidir_attention(q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens,
                                        scale=D**-0.5)
        ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
        assert float((out.float().cpu() - ref).abs().max()) <= TOL, (B, S)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("B,H,Hkv,S,L,D,dtype,seed", [(300, 4, 2, 200, 40, 32, torch.bfloat16, 41),
                                                       (64, 16, 4, 1000, 260, 64, torch.float16, 42),
                                                       (150, 8, 8, 300, 130, 128, torch.bfloat16, 43)])
def test_persistent_units_ragged_against_oracle(B, H, Hkv, S, L, D, dtype, seed):
    """More units than SMs, so every CTA of the persistent launch walks several
    units: empty blocks (units with no key tile) between full ones, blocks of
    one to three own key tiles (units of different lengths in one CTA's
    sequence), an odd number of key tiles per unit (the softmax groups swap
    roles from one unit to the next), fp16, G in {1, 2, 4}. Two launches give
    the same bits."""
    g = torch.Generator().manual_seed(seed)
    q = _rand((B, H, L, D), g, dtype)
    ks, vs = _rand((Hkv, S, D), g, dtype), _rand((Hkv, S, D), g, dtype)
    kq, vq = _rand((B, Hkv, L, D), g, dtype), _rand((B, Hkv, L, D), g, dtype)
    lens = torch.randint(0, L + 1, (B,), generator=g)
    lens[::7] = 0
    lens[1::5] = L
    lens = lens.tolist()
    args = (q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens)
    out = pb.prefix_bidir_attention(*args, scale=D**-0.5)
    out_again = pb.prefix_bidir_attention(*args, scale=D**-0.5)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(out, out_again)
    ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
    got = out.float().cpu()
    assert float((got - ref).abs().max()) <= TOL
    for b, n in enumerate(lens):
        assert bool((got[b, :, n:] == 0).all())


@pytest.mark.parametrize("B,H,Hkv,S,L,dtype,seed", [(40, 32, 4, 1000, 64, torch.bfloat16, 51),
                                                     (160, 16, 2, 300, 128, torch.float16, 52)])
def test_cta_pair_kernel_ragged_against_oracle(B, H, Hkv, S, L, dtype, seed):
    """Shapes the CTA-pair kernel serves (head_dim 128, an even number of Q tiles
    per block and kv head, at least four units per SM, no cut tail): ragged
    blocks where the upper Q tile of a pair holds no real token while the lower
    one does (its rows are computed and written as zeros), pairs with no real
    token at all, empty blocks, fp16 and bf16. Two launches give the same bits."""
    D = 128
    g = torch.Generator().manual_seed(seed)
    q = _rand((B, H, L, D), g, dtype)
    ks, vs = _rand((Hkv, S, D), g, dtype), _rand((Hkv, S, D), g, dtype)
    kq, vq = _rand((B, Hkv, L, D), g, dtype), _rand((B, Hkv, L, D), g, dtype)
    T = 128 // (H // Hkv)
    lens = torch.randint(0, L + 1, (B,), generator=g)
    lens[::5] = 2 * T + 3   # the pair (tiles 2, 3): lower tile partly real, upper tile empty
    lens[1::7] = T - 1      # the pair (tiles 0, 1): upper tile empty; later pairs empty
    lens[2::9] = 0
    lens[3::11] = L
    lens = lens.tolist()
    args = (q.to(DEV), ks.to(DEV), vs.to(DEV), kq.to(DEV), vq.to(DEV), lens)
    out = pb.prefix_bidir_attention(*args, scale=D**-0.5)
    out_again = pb.prefix_bidir_attention(*args, scale=D**-0.5)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(out, out_again)
    ref = oattn.questions(q, ks, vs, kq, vq, lens, D**-0.5, dtype=torch.float32)
    got = out.float().cpu()
    assert float((got - ref).abs().max()) <= TOL
    for b, n in enumerate(lens):
        assert bool((got[b, :, n:] == 0).all())
