"""Config 4 end to end on B200: the reduced backbone of tests/e2e_model.py through
D3Backbone (state pass, question pass, 255-way readout on this library's kernels)
against the reference's own D3Core run on transformers' Qwen3.5 layers with its
FP8 QuantLinear (tests/golden/e2e_4layer.npz, tests/golden/make_e2e_golden.py).

The gate is the reference's parity rule (d3trt/parity.py:29, :128-182): every
per-answer probability within 1e-2 and the same argmax for every block. The
question pass on a snapshot packed into the cache's arena format gives the same
bits as on the state pass's own tensors."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import e2e_model as em
from conftest import load_golden

from d3_turbo_trt_b200 import _lib
from d3_turbo_trt_b200.model.backbone import BackboneConfig, D3Backbone

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
PROB_TOL = 1e-2


def _run(gdn_state="ours"):
    bb = D3Backbone(BackboneConfig(**em.CONFIG), em.make_weights(), device=DEV, mode="fp8", gdn_state=gdn_state)
    state, ids, lengths, counts, readout = em.make_request()
    snap = bb.state(state)
    hidden = bb.questions(snap, ids, lengths, state_len=state.shape[1])
    probs = bb.probabilities(hidden, readout.to(DEV), counts)
    return bb, snap, (state, ids, lengths, counts, readout), hidden, probs


def _check(probs, hidden):
    g = load_golden("e2e_4layer.npz")
    got = probs.cpu().numpy()
    ref = g["probs"]
    for r, n in enumerate(g["counts"]):
        assert np.all(got[r, n:] == 0)
    diff = np.abs(got - ref).max()
    assert diff <= PROB_TOL, diff
    assert np.array_equal(got.argmax(1), ref.argmax(1))
    return diff, float(np.abs(hidden.float().cpu().numpy() - g["hidden"]).max())


def test_end_to_end_readout_matches_reference_d3core():
    bb, snap, req, hidden, probs = _run()
    _check(probs, hidden)
    # the same question pass on the snapshot packed into the state cache's format
    from d3_turbo_trt_b200.model.snapshot import SnapshotArena, pack_snapshot

    state, ids, lengths, counts, readout = req
    arena = SnapshotArena(64 << 20, DEV)
    packed = pack_snapshot(snap, arena)
    hidden2 = bb.questions(packed, ids, lengths, state_len=state.shape[1])
    assert torch.equal(hidden2, hidden)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_end_to_end_with_fla_state_scan():
    pytest.importorskip("fla.ops.gated_delta_rule")
    _, _, _, hidden, probs = _run(gdn_state="fla")
    _check(probs, hidden)
