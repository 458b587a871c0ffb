"""QuestionPipeline (overlapped copy in / question pass / copy out) gives the
same outputs as calling prefix_bidir_attention on each batch in turn."""

from __future__ import annotations

import pytest
import torch

from d3_turbo_trt_b200.kernels import prefix_bidir as pb
from d3_turbo_trt_b200.kernels.pipeline import QuestionPipeline

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_pipeline_matches_per_batch_calls():
    g = torch.Generator().manual_seed(7)
    B, H, Hkv, L, D, S = 6, 8, 2, 40, 64, 300
    ks = torch.randn(Hkv, S, D, generator=g).to(torch.bfloat16).to(DEV)
    vs = torch.randn(Hkv, S, D, generator=g).to(torch.bfloat16).to(DEV)
    batches, want = [], []
    for i in range(5):  # more batches than pipeline slots, different lengths per batch
        q = torch.randn(B, H, L, D, generator=g).to(torch.bfloat16).pin_memory()
        kq = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16).pin_memory()
        vq = torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16).pin_memory()
        lens = [(7 * i + 5 * b) % L + 1 for b in range(B)]
        out = torch.full((B, H, L, D), 7.0, dtype=torch.bfloat16).pin_memory()
        batches.append((q, kq, vq, lens, out))
        want.append(pb.prefix_bidir_attention(q.to(DEV), ks, vs, kq.to(DEV), vq.to(DEV), lens, scale=D ** -0.5).cpu())
    pipe = QuestionPipeline(ks, vs, scale=D ** -0.5, depth=2)
    events = [pipe.submit(*b) for b in batches]
    pipe.synchronize()
    for e in events:
        assert e.query()
    for (_, _, _, _, out), w in zip(batches, want):
        assert torch.equal(out, w)


def test_graph_replay_matches_eager_pipeline():
    """Pinned host buffers take the graph path: one captured graph per (slot, host
    buffers, lengths); replays with new data in the same buffers, a change of
    lengths (a new capture) and buffers alternating between slots give the same
    bits as the eager pipeline. wait_stream/join bracket the work for timing."""
    g = torch.Generator().manual_seed(11)
    B, H, Hkv, L, D, S = 16, 32, 4, 64, 128, 1024
    ks = torch.randn(Hkv, S, D, generator=g).to(torch.bfloat16).to(DEV)
    vs = torch.randn(Hkv, S, D, generator=g).to(torch.bfloat16).to(DEV)
    bufs = [tuple(torch.empty(*shp, dtype=torch.bfloat16).pin_memory() for shp in
                  ((B, H, L, D), (B, Hkv, L, D), (B, Hkv, L, D), (B, H, L, D))) for _ in range(2)]
    graph_pipe = QuestionPipeline(ks, vs, scale=D ** -0.5, depth=2, graphs=True)
    eager_pipe = QuestionPipeline(ks, vs, scale=D ** -0.5, depth=2)
    cur = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for step in range(7):
        q, kq, vq, out = bufs[step % 2]
        q.copy_(torch.randn(B, H, L, D, generator=g).to(torch.bfloat16))
        kq.copy_(torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16))
        vq.copy_(torch.randn(B, Hkv, L, D, generator=g).to(torch.bfloat16))
        lens = [L] * B if step < 4 else [(5 * b + 3) % L + 1 for b in range(B)]
        ref = torch.empty_like(out)  # pageable: the eager pipeline's path
        eager_pipe.submit(q, kq, vq, lens, ref)
        eager_pipe.synchronize()
        start.record(cur)
        graph_pipe.wait_stream(cur)
        ev = graph_pipe.submit(q, kq, vq, lens, out)
        graph_pipe.join(cur)
        end.record(cur)
        ev.synchronize()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), step
        assert start.elapsed_time(end) > 0
    assert len(graph_pipe._graphs) == 4  # (slot, buffers) x {full, ragged lengths}
