"""Question-pass scheduling (kernels/graphs.py): the reference's batch bounds
(reference/d3_runtime.py:1290-1314) on CPU, and CUDA-graph replay of the
question pass against eager calls on the GPU."""

from __future__ import annotations

import random

import pytest
import torch

from d3_turbo_trt_b200.kernels import graphs


def test_state_once_batches_bounds_and_order():
    rng = random.Random(0)
    for state in (0, 512, 4096, 16384, 200000):
        lengths = [rng.randint(1, 300) for _ in range(257)]
        batches = graphs.state_once_batches(lengths, state)
        flat = [i for b in batches for i in b]
        assert sorted(flat) == list(range(len(lengths)))  # every block exactly once
        assert [lengths[i] for i in flat] == sorted(lengths)  # shortest first
        for b in batches:
            rows, widest = len(b), max(lengths[i] for i in b)
            if rows > 1:  # a block too large for the bounds gets a batch of its own
                assert rows <= graphs.STATE_ONCE_ROWS
                assert rows * (state + widest) <= graphs.STATE_ONCE_KEYS
                assert rows * widest * (state + widest) <= graphs.STATE_ONCE_SCORES
        # greedy: the next block would have broken a bound of each closed batch
        for b, nxt in zip(batches, batches[1:]):
            rows, widest = len(b) + 1, lengths[nxt[0]]
            assert (rows > graphs.STATE_ONCE_ROWS or rows * (state + widest) > graphs.STATE_ONCE_KEYS
                    or rows * widest * (state + widest) > graphs.STATE_ONCE_SCORES)


def test_single_batch():
    assert graphs.single_batch([]) == []
    assert graphs.single_batch([5, 2, 9, 2]) == [[1, 3, 0, 2]]


@pytest.mark.gpu
def test_graph_replay_matches_eager():
    from d3_turbo_trt_b200.kernels import prefix_bidir as pb

    g = torch.Generator().manual_seed(3)
    R, H, Hkv, W, D, S = 7, 16, 2, 48, 128, 700
    ks = torch.randn(Hkv, S, D, generator=g).to(torch.bfloat16).cuda()
    vs = torch.randn(Hkv, S, D, generator=g).to(torch.bfloat16).cuda()
    gp = graphs.QuestionPassGraph(ks, vs, rows=R, width=W, heads=H, scale=D ** -0.5)
    for trial in range(3):
        q = torch.randn(R, H, W, D, generator=g).to(torch.bfloat16).cuda()
        kq = torch.randn(R, Hkv, W, D, generator=g).to(torch.bfloat16).cuda()
        vq = torch.randn(R, Hkv, W, D, generator=g).to(torch.bfloat16).cuda()
        lens = [(11 * trial + 7 * r) % W + 1 for r in range(R)]
        got = gp.run(q, kq, vq, lens if trial != 1 else torch.tensor(lens, dtype=torch.int32).cuda()).clone()
        want = pb.prefix_bidir_attention(q, ks, vs, kq, vq, lens, scale=D ** -0.5)
        assert torch.equal(got, want)
