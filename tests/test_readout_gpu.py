"""GPU parity of the 255-way readout against the golden vectors recorded from
TrtllmStack.probabilities (trtllm_stack.py:451-468) and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_from_bits, load_golden
from oracle import readout as oread

import d3_turbo_trt_b200 as d3b

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("tag", ["t1", "t07"])
def test_readout_golden(tag):
    g = load_golden("readout.npz")
    hidden = bf16_from_bits(g["hidden_bf16"]).to(DEV)
    readout = torch.from_numpy(g["readout"]).to(DEV)
    counts = g["counts"].tolist()
    temp = float(g[f"temp_{tag}"])
    lists = d3b.probabilities(hidden, readout, counts, temperature=temp)
    assert [len(r) for r in lists] == counts
    for row, ref in zip(lists, g[f"probs_{tag}"]):
        assert np.abs(np.array(row) - ref[: len(row)]).max() <= 1e-5


def test_readout_cfg4_shape_twice():
    """255 blocks x hidden 5120 x 255 options; two calls in a row reuse the workspace."""
    g = torch.Generator().manual_seed(21)
    hidden = torch.randn(255, 5120, generator=g).to(torch.bfloat16)
    readout = torch.randn(255, 5120, generator=g) * 0.02
    counts = [1 + (i * 37) % 255 for i in range(255)]
    ref = oread.probabilities(hidden.float().numpy(), readout.numpy(), counts, 1.0)
    for _ in range(2):
        probs = d3b.probabilities_tensor(hidden.to(DEV), readout.to(DEV), counts, temperature=1.0).cpu().numpy()
        assert np.abs(probs - ref).max() <= 1e-5
        assert np.argmax(probs, 1).tolist() == np.argmax(ref, 1).tolist()


def test_readout_odd_sizes():
    g = torch.Generator().manual_seed(22)
    for rows, k, n_opt in ((1, 100, 3), (9, 777, 40), (33, 512, 1000)):
        hidden = torch.randn(rows, k, generator=g)
        readout = torch.randn(n_opt, k, generator=g) * 0.05
        counts = [(i % n_opt) + 1 for i in range(rows)]
        ref = oread.probabilities(hidden.numpy(), readout.numpy(), counts, 0.5)
        got = d3b.probabilities_tensor(hidden.to(DEV), readout.to(DEV), counts, temperature=0.5).cpu().numpy()
        assert np.abs(got - ref).max() <= 1e-5


def test_readout_planes_path_against_fp32_path():
    """bf16 hidden rows take the tensor-core path (the fp32 readout split into three bf16
    planes, exact products, fp32 accumulation): within 1e-5 of the oracle and of the fp32
    FMA path (fp32 hidden of the same values), including the model's shape, rows past one
    128-row tile, options past 256, counts of 1 and n_opt, and a K that is not a multiple
    of the 64-wide K chunk; an in-place change of the readout makes new planes."""
    from d3_turbo_trt_b200.model import readout as ro

    g = torch.Generator().manual_seed(23)
    for rows, k, n_opt in ((255, 5120, 255), (130, 1000, 300), (3, 64, 1), (200, 5128, 1024)):
        hidden = torch.randn(rows, k, generator=g).to(torch.bfloat16)
        readout = torch.randn(n_opt, k, generator=g) * 0.02
        counts = [1 + (i * 37) % n_opt for i in range(rows)]
        counts[0] = n_opt
        ref = oread.probabilities(hidden.float().numpy(), readout.numpy(), counts, 0.7)
        rd = readout.to(DEV)
        got = d3b.probabilities_tensor(hidden.to(DEV), rd, counts, temperature=0.7)
        fp32 = d3b.probabilities_tensor(hidden.float().to(DEV), rd, counts, temperature=0.7)
        assert np.abs(got.cpu().numpy() - ref).max() <= 1e-5, (rows, k, n_opt)
        assert float((got - fp32).abs().max()) <= 1e-5
        assert np.argmax(got.cpu().numpy(), 1).tolist() == np.argmax(ref, 1).tolist()
    # planes follow in-place updates of the readout matrix
    hidden = torch.randn(8, 256, generator=g).to(torch.bfloat16).to(DEV)
    rd = (torch.randn(16, 256, generator=g) * 0.05).to(DEV)
    first = d3b.probabilities_tensor(hidden, rd, [16] * 8, temperature=1.0)
    rd.mul_(-1.0)
    second = d3b.probabilities_tensor(hidden, rd, [16] * 8, temperature=1.0)
    ref = oread.probabilities(hidden.float().cpu().numpy(), rd.cpu().numpy(), [16] * 8, 1.0)
    assert np.abs(second.cpu().numpy() - ref).max() <= 1e-5
    assert not torch.equal(first, second)
    assert len(ro._PLANES) <= 4


def test_readout_planes_not_reused_for_a_new_matrix_at_a_freed_address():
    """A readout matrix freed and a new one of the same shape allocated in its place (the
    caching allocator hands the same block back) gets its own planes, not the freed one's."""
    g = torch.Generator().manual_seed(31)
    hidden = torch.randn(16, 512, generator=g).to(torch.bfloat16).to(DEV)
    counts = [40] * 16
    rd = (torch.randn(40, 512, generator=g) * 0.05).to(DEV)
    d3b.probabilities_tensor(hidden, rd, counts, temperature=1.0)
    addr = rd.data_ptr()
    del rd
    rd = (torch.randn(40, 512, generator=g) * 0.05).to(DEV)
    got = d3b.probabilities_tensor(hidden, rd, counts, temperature=1.0)
    ref = oread.probabilities(hidden.float().cpu().numpy(), rd.cpu().numpy(), counts, 1.0)
    assert np.abs(got.cpu().numpy() - ref).max() <= 1e-5, ("same address" if rd.data_ptr() == addr else "moved")
