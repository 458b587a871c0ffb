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
