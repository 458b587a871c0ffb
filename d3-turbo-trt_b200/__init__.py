"""d3-turbo-trt on B200: sm_100a kernels for the d3 prefill hot path.

Drop-in operators with the reference signatures (pramodsarvi/d3-turbo-trt):

* ``kernels.prefix_bidir.prefix_bidir_attention`` and ``state_attention`` —
  prefix-bidirectional GQA attention (tcgen05 + TMA + TMEM);
* ``model.quant`` — ``quantize_rows``, ``quantize_weight``, ``QuantLinear``
  (W8A8 e4m3 / int8 on tcgen05 with fused dequant epilogue);
* ``model.readout.probabilities`` — the 255-way fp32 readout softmax;
* ``dist`` — state-KV broadcast and question-block sharding over NCCL.

All compute goes through ``libd3b200.so`` (C ABI in ``include/d3b200.h``).
"""

from . import _lib
from .kernels.prefix_bidir import prefix_bidir_attention, state_attention
from .model.quant import QuantLinear, make_linear, quantize_rows, quantize_weight, scaled_mm
from .model.readout import ReadoutHead, probabilities, probabilities_tensor

__version__ = "0.1.0"

__all__ = [
    "QuantLinear",
    "ReadoutHead",
    "make_linear",
    "prefix_bidir_attention",
    "probabilities",
    "probabilities_tensor",
    "quantize_rows",
    "quantize_weight",
    "scaled_mm",
    "state_attention",
]
