"""QuestionBatcher against the reference backend's id construction
(d3trt/backends/trtllm.py:149-162, restated below as the check): the same
batches in the same order, the same padded int64 ids, the same lengths."""

from __future__ import annotations

import random

import pytest
import torch

from d3_turbo_trt_b200.model.batching import QuestionBatcher, batch_orders


def _reference_batches(pieces, batch_size, pad_id, device):
    order = sorted(range(len(pieces)), key=lambda i: len(pieces[i]))
    size = max(1, int(batch_size))
    out = []
    for start in range(0, len(order), size):
        batch = order[start:start + size]
        rows = [pieces[i] for i in batch]
        width = max(map(len, rows))
        ids = torch.full((len(rows), width), pad_id, dtype=torch.long, device=device)
        for r, piece in enumerate(rows):
            ids[r, :len(piece)] = torch.as_tensor(piece, dtype=torch.long, device=device)
        out.append((batch, ids, [len(p) for p in rows]))
    return out


def _pieces(seed, n, lo=0, hi=64, vocab=151_936):
    rng = random.Random(seed)
    return [[rng.randrange(vocab) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


def _check(device, pieces, batch_size, pad_id=0):
    ref = _reference_batches(pieces, batch_size, pad_id, device)
    got = list(QuestionBatcher(device, pad_id).batches(pieces, batch_size))
    assert len(got) == len(ref)
    for g, (index, ids, lens) in zip(got, ref):
        assert g.index == index
        assert g.lengths == lens
        assert g.ids.dtype == torch.int64 and g.ids.device.type == torch.device(device).type
        assert torch.equal(g.ids, ids)
        assert g.lengths_dev.tolist() == lens


@pytest.mark.parametrize("batch_size", [1, 7, 64, 255, 1000])
def test_batches_match_reference_cpu(batch_size):
    _check("cpu", _pieces(1, 255, 1, 48), batch_size, pad_id=151_643)


def test_ties_keep_request_order_and_empty_pieces():
    pieces = [[5, 6], [], [7, 8], [1], [], [9, 9, 9]]
    assert batch_orders(pieces, 2) == [[1, 4], [3, 0], [2, 5]]
    _check("cpu", pieces, 2)
    _check("cpu", [[], []], 4)  # every piece empty: [rows, 0] ids


def test_staging_reuse_keeps_earlier_batches():
    b = QuestionBatcher("cpu", 0)
    first = b.build([[1, 2, 3], [4]])
    b.build([[9] * 50])
    b.build([[8] * 10, [7] * 3])
    assert first[0].tolist() == [[1, 2, 3], [4, 0, 0]] and first[1].tolist() == [3, 1]


@pytest.mark.gpu
@pytest.mark.parametrize("batch_size", [1, 16, 255])
def test_batches_match_reference_gpu(batch_size):
    pieces = _pieces(2, 255, 1, 48)
    _check("cuda", pieces, batch_size, pad_id=151_643)
    # many batches in flight: the two pinned staging buffers rotate under non-blocking copies
    b = QuestionBatcher("cuda", 0)
    built = [b.build(_pieces(10 + i, 33, 0, 64)) for i in range(12)]
    torch.cuda.synchronize()
    for i, (ids, lens) in enumerate(built):
        rows = _pieces(10 + i, 33, 0, 64)
        assert lens.tolist() == [len(r) for r in rows]
        assert ids.tolist() == [r + [0] * (ids.shape[1] - len(r)) for r in rows]
