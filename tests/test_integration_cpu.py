"""The drop-in rebinding applied to the reference package itself (CPU, no GPU).

Imports the reference's d3trt (skipped where it is not on this machine), runs
d3_turbo_trt_b200.integration.install() and checks that every name the
reference's D3Core, quantised linears, stacks and backend look up at call time
now resolves to this library, then puts the originals back. D3Core reaches its
attention and GDN kernels through the ops module (d3trt/model/core.py:253-265,
:360-372), so these are exactly the objects its next call uses."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

# the reference checkout: D3_REFERENCE_DIR, else a `reference` folder beside this repository
REF = Path(os.environ.get("D3_REFERENCE_DIR", Path(__file__).resolve().parents[2] / "reference"))


@pytest.fixture
def d3trt():
    if not (REF / "d3trt").is_dir():
        pytest.skip("the reference package is not on this machine")
    sys.path.insert(0, str(REF))
    try:
        import d3trt  # noqa: F401

        yield
    finally:
        sys.path.remove(str(REF))


def test_install_rebinds_every_hot_path_name(d3trt):
    from d3trt.kernels import prefix_bidir as ref_attn
    from d3trt.model import core as ref_core
    from d3trt.model import ops as ref_ops
    from d3trt.model import quant as ref_quant

    from d3_turbo_trt_b200 import integration
    from d3_turbo_trt_b200.kernels import prefix_bidir as attn
    from d3_turbo_trt_b200.model import gdn, ops, quant

    originals = {"qa": ref_ops.question_attention, "ql": ref_quant.QuantLinear}
    previous = integration.install()
    try:
        assert ref_attn.prefix_bidir_attention is attn.prefix_bidir_attention
        assert ref_ops.question_attention is ops.question_attention
        assert ref_ops.flash_state is ops.flash_state
        assert ref_ops.recurrent_gated_delta_rule is gdn.question_gated_delta_rule
        assert ref_ops.chunk_gated_delta_rule is gdn.chunk_gated_delta_rule
        assert ref_quant.QuantLinear is quant.QuantLinear
        assert ref_quant.make_linear is quant.make_linear
        assert ref_quant.quantize_rows is quant.quantize_rows
        # D3Core looks its kernels up through the module at call time
        assert ref_core.ops is ref_ops
        try:
            from d3trt.model import trtllm_stack as ref_stack
        except Exception:  # noqa: BLE001
            ref_stack = None
        if ref_stack is not None:
            assert ref_stack.QuantLinear is quant.QuantLinear
            assert ref_stack.TrtllmStack.probabilities is not None
            assert "d3_turbo_trt_b200" in ref_stack.TrtllmStack.probabilities.__module__
        # our drop-ins keep the reference's error behaviour: a CPU tensor raises RuntimeError
        import torch

        with pytest.raises(RuntimeError):
            ref_attn.prefix_bidir_attention(torch.zeros(1, 2, 4, 64), torch.zeros(1, 8, 64), torch.zeros(1, 8, 64),
                                            torch.zeros(1, 1, 4, 64), torch.zeros(1, 1, 4, 64), [4], scale=0.125)
    finally:
        integration.uninstall(previous)
    assert ref_ops.question_attention is originals["qa"]
    assert ref_quant.QuantLinear is originals["ql"]
