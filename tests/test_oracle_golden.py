"""Pin the CPU oracle to the reference: every oracle function against the golden
vectors that tests/golden/make_golden.py recorded from the reference's own code.
Also restates the reference's own quant tests (tests/test_quant.py) on the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import attention as oattn
from oracle import quant as oq
from oracle import readout as oread


@pytest.fixture(scope="module")
def gq():
    return load_golden("quant.npz")


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_quantize_rows_bf16_bit_exact(gq, mode):
    x = bf16_from_bits(gq["rows_x_bf16"]).float().numpy()
    q, s = oq.quantize_rows(x, mode)
    assert np.array_equal(s, gq[f"rows_s_{mode}"])
    assert np.array_equal(q.view(np.uint8), gq[f"rows_q_{mode}"].view(np.uint8))


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_quantize_rows_f32_bit_exact(gq, mode):
    q, s = oq.quantize_rows(gq["rows_x_f32"], mode)
    assert np.array_equal(s, gq[f"rows32_s_{mode}"])
    assert np.array_equal(q.view(np.uint8), gq[f"rows32_q_{mode}"].view(np.uint8))


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_quantize_weight_bit_exact(gq, mode):
    w = bf16_from_bits(gq["w_bf16"]).float().numpy()
    q, s = oq.quantize_weight(w, mode)
    assert np.array_equal(s, gq[f"w_s_{mode}"])
    assert np.array_equal(q.view(np.uint8), gq[f"w_q_{mode}"].view(np.uint8))


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_w8a8_linear_matches_emulated(gq, mode):
    x = bf16_from_bits(gq["lin_x_bf16"]).float().numpy().reshape(-1, 256)
    w = bf16_from_bits(gq["w_bf16"]).float().numpy()
    qa, sa = oq.quantize_rows(x, mode)
    qw, sw = oq.quantize_weight(w, mode)
    if mode == "int8":
        assert np.array_equal(oq.int_gemm(qa, qw).astype(np.float32), gq["lin_acc_int8"])
    y = oq.w8a8_linear(qa, sa, qw, sw, mode)
    np.testing.assert_allclose(y, gq[f"lin_f32_{mode}"], rtol=2e-6, atol=1e-7)
    ref_bf16 = bf16_from_bits(gq[f"lin_y_{mode}_bf16"]).float().numpy().reshape(y.shape)
    mine = oq.bf16_round(y)
    if mode == "int8":
        assert np.array_equal(mine, ref_bf16)
    else:  # fp32 summation order may move a value across a bf16 rounding boundary
        assert np.mean(mine != ref_bf16) < 1e-3


def test_e4m3_round_trip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    vals = oq.e4m3_decode(codes)
    finite = ~np.isnan(vals)
    assert np.array_equal(oq.e4m3_encode(vals[finite]), codes[finite])


def test_e4m3_encoder_matches_torch_cast():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 60, 100_000), rng.normal(0, 0.01, 100_000)]).astype(np.float32)
    x = np.clip(x, -448, 448)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(oq.e4m3_encode(x), ref)


# --- the reference's own quant tests (tests/test_quant.py:15-50), on the oracle ---


@pytest.mark.parametrize("mode,limit", [("fp8", 0.06), ("int8", 0.02)])
def test_quant_linear_matches_dense(mode, limit):
    torch.manual_seed(0)
    weight = torch.randn(96, 256) * 0.02
    x = torch.randn(3, 5, 256, dtype=torch.bfloat16)
    wq, ws = oq.quantize_weight(weight.to(torch.bfloat16).float().numpy(), mode)
    qa, sa = oq.quantize_rows(x.float().numpy().reshape(-1, 256), mode)
    out = oq.bf16_round(oq.w8a8_linear(qa, sa, wq, ws, mode))
    ref = (x.float() @ weight.t()).numpy().reshape(-1, 96)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < limit


def test_per_token_scale_handles_outlier_rows_and_zero_rows():
    torch.manual_seed(0)
    weight = torch.randn(32, 64)
    x = torch.randn(4, 64)
    x[1] *= 1000.0
    x[3] = 0.0
    wq, ws = oq.quantize_weight(weight.numpy(), "int8")
    qa, sa = oq.quantize_rows(x.numpy(), "int8")
    out = oq.w8a8_linear(qa, sa, wq, ws, "int8")
    ref = (x @ weight.t()).numpy()
    assert np.linalg.norm(out[0] - ref[0]) / np.linalg.norm(ref[0]) < 0.02
    assert np.all(out[3] == 0)


def test_weight_quantization_is_per_channel():
    weight = np.ones((16, 32), dtype=np.float32)
    weight[0] *= 100.0
    q, scale = oq.quantize_weight(weight, "int8")
    assert q.dtype == np.int8 and scale.shape == (16,)
    assert np.all(q == 127)
    assert scale[0] == pytest.approx(100.0 / 127)
    assert scale[1] == pytest.approx(1.0 / 127)


# --- attention ---


def _cfg1():
    g = load_golden("attn_cfg1.npz")
    state, nb, lq, heads, kv_heads, dim = (int(v) for v in g["meta"])
    Q = bf16_from_bits(g["Q"]).float()
    K = bf16_from_bits(g["K"]).float()
    V = bf16_from_bits(g["V"]).float()
    return g, state, nb, lq, heads, kv_heads, dim, Q, K, V


def test_attention_cfg1_question_and_state_pass():
    g, state, nb, lq, heads, kv_heads, dim, Q, K, V = _cfg1()
    scale = float(g["scale"])
    ks, vs = K[:state].transpose(0, 1), V[:state].transpose(0, 1)
    out_state = oattn.state(Q[:state].transpose(0, 1)[None], ks[None], vs[None], scale)[0].transpose(0, 1)
    qq = Q[state:].view(nb, lq, heads, dim).permute(0, 2, 1, 3)
    kq = K[state:].view(nb, lq, kv_heads, dim).permute(0, 2, 1, 3)
    vq = V[state:].view(nb, lq, kv_heads, dim).permute(0, 2, 1, 3)
    out_q = oattn.questions(qq, ks, vs, kq, vq, [lq] * nb, scale)
    out = torch.cat([out_state, out_q.permute(0, 2, 1, 3).reshape(nb * lq, heads, dim)], 0)
    np.testing.assert_allclose(out.numpy(), g["out"], atol=2e-6, rtol=0)


def test_attention_cfg1_dense_mask_semantics():
    g, state, nb, lq, heads, kv_heads, dim, Q, K, V = _cfg1()
    out = oattn.masked_sequence(Q, K, V, state, [lq] * nb, float(g["scale"]))
    np.testing.assert_allclose(out.numpy(), g["out"], atol=2e-6, rtol=0)


@pytest.mark.parametrize("case", ["d32_g2", "d64_g3", "d256_g1", "d128_g8"])
def test_attention_ragged(case):
    g = load_golden("attn_ragged.npz")
    t = {k: bf16_from_bits(g[f"{case}_{k}"]).float() for k in ("q", "ks", "vs", "kq", "vq")}
    out = oattn.questions(t["q"], t["ks"], t["vs"], t["kq"], t["vq"], g[f"{case}_lens"].tolist(),
                          float(g[f"{case}_scale"]))
    np.testing.assert_allclose(out.numpy(), g[f"{case}_out"], atol=2e-6, rtol=0)
    # the reference's own call pattern (timed by bench.py's reference arm) gives the golden too
    out = oattn.questions_sdpa(t["q"], t["ks"], t["vs"], t["kq"], t["vq"], g[f"{case}_lens"].tolist(),
                               float(g[f"{case}_scale"]))
    np.testing.assert_allclose(out.numpy(), g[f"{case}_out"], atol=2e-6, rtol=0)


# --- readout ---


@pytest.mark.parametrize("tag", ["t1", "t07"])
def test_readout(tag):
    g = load_golden("readout.npz")
    hidden = bf16_from_bits(g["hidden_bf16"]).float().numpy()
    probs = oread.probabilities(hidden, g["readout"], g["counts"], float(g[f"temp_{tag}"]))
    np.testing.assert_allclose(probs, g[f"probs_{tag}"], atol=1e-6, rtol=1e-5)
    lists = oread.probabilities_lists(hidden, g["readout"], g["counts"], float(g[f"temp_{tag}"]))
    assert [len(r) for r in lists] == g["counts"].tolist()
