"""Drop this library into an imported d3trt (the reference package) by rebinding.

``install()`` replaces, in the caller's ``d3trt`` modules, every function and class
on the hot path with this library's drop-in of the same signature, so the
reference's own scheduler, ``D3Core`` (d3trt/model/core.py:146-402), state cache
and stacks run on the sm_100a kernels unchanged:

=====================================================  ======================================
d3trt name (file:line)                                 replaced by
=====================================================  ======================================
kernels/prefix_bidir.py:187 ``prefix_bidir_attention``  kernels.prefix_bidir.prefix_bidir_attention
kernels/prefix_bidir.py ``triton_available``            kernels.prefix_bidir.kernel_available
model/ops.py:227 ``question_attention``                 model.ops.question_attention
model/ops.py:174 ``flash_state``                        model.ops.flash_state
model/ops.py:327 ``recurrent_gated_delta_rule``         model.gdn.question_gated_delta_rule
model/ops.py:287 ``chunk_gated_delta_rule``             model.gdn.chunk_gated_delta_rule
model/quant.py ``quantize_rows``, ``quantize_weight``,  model.quant (same names)
``QuantLinear``, ``make_linear``
model/trtllm_stack.py ``QuantLinear``, ``make_linear``  model.quant (same names)
model/trtllm_stack.py:451 ``TrtllmStack.probabilities``  model.readout.ReadoutHead(readout).probabilities
backends/trtllm.py ``StateCache``                       model.cache.StateCache with an arena
=====================================================  ======================================

``D3Core`` calls the ops through the module (``ops.question_attention(...)``), so
rebinding the module attributes is enough; nothing in d3trt is edited.
"""

from __future__ import annotations

import importlib
import types
from typing import Any

from .kernels import prefix_bidir as _attn
from .model import gdn as _gdn
from .model import ops as _ops
from .model import quant as _quant
from .model.readout import ReadoutHead


def _stack_probabilities(self, hidden, counts, *, temperature, readout_dtype="float32"):
    return ReadoutHead(self.readout).probabilities(hidden, counts, temperature=temperature,
                                                   readout_dtype=readout_dtype)


def _state_cache(budget: int):
    from .model.cache import StateCache
    from .model.snapshot import SnapshotArena

    return StateCache(budget, arena=SnapshotArena(budget + (64 << 20)))


def install(package: str = "d3trt", *, cache: bool = True) -> dict[str, Any]:
    """Rebind d3trt's hot-path names to this library; returns {qualified name: previous object}
    so a caller (a test) can put them back. Modules that d3trt cannot import on this machine
    (the TRT-LLM stack without tensorrt_llm) are skipped, never partly patched."""
    previous: dict[str, Any] = {}

    def bind(owner, name, value):
        prefix = owner.__name__ if isinstance(owner, types.ModuleType) else f"{owner.__module__}.{owner.__qualname__}"
        previous[f"{prefix}.{name}"] = getattr(owner, name)
        setattr(owner, name, value)

    ref_attn = importlib.import_module(f"{package}.kernels.prefix_bidir")
    ref_ops = importlib.import_module(f"{package}.model.ops")
    ref_quant = importlib.import_module(f"{package}.model.quant")
    bind(ref_attn, "prefix_bidir_attention", _attn.prefix_bidir_attention)
    bind(ref_attn, "triton_available", _attn.kernel_available)
    bind(ref_ops, "question_attention", _ops.question_attention)
    bind(ref_ops, "flash_state", _ops.flash_state)
    bind(ref_ops, "recurrent_gated_delta_rule", _gdn.question_gated_delta_rule)
    bind(ref_ops, "chunk_gated_delta_rule", _gdn.chunk_gated_delta_rule)
    for name in ("quantize_rows", "quantize_weight", "QuantLinear", "make_linear"):
        bind(ref_quant, name, getattr(_quant, name))
    try:
        ref_stack = importlib.import_module(f"{package}.model.trtllm_stack")
    except Exception:  # noqa: BLE001 - optional module of the reference
        ref_stack = None
    if ref_stack is not None:
        bind(ref_stack, "QuantLinear", _quant.QuantLinear)
        bind(ref_stack, "make_linear", _quant.make_linear)
        bind(ref_stack.TrtllmStack, "probabilities", _stack_probabilities)
    if cache:
        try:
            ref_backend = importlib.import_module(f"{package}.backends.trtllm")
        except Exception:  # noqa: BLE001
            ref_backend = None
        if ref_backend is not None and hasattr(ref_backend, "StateCache"):
            bind(ref_backend, "StateCache", _state_cache)
    return previous


def uninstall(previous: dict[str, Any]) -> None:
    """Put back what ``install`` replaced."""
    for qual, value in previous.items():
        mod_name, _, name = qual.rpartition(".")
        try:
            owner = importlib.import_module(mod_name)
        except ModuleNotFoundError:  # a class attribute: module.Class.name
            mod_name, _, cls = mod_name.rpartition(".")
            owner = getattr(importlib.import_module(mod_name), cls)
        setattr(owner, name, value)
