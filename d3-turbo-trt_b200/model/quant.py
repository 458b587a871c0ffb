"""W8A8 quantised Linear on the sm_100a kernels (drop-in for d3trt/model/quant.py).

Same public surface as the reference module: ``MODES``, ``fp8_supported``,
``resolve_mode``, ``quantizable``, ``quantize_weight``, ``quantize_rows``,
``QuantLinear`` (``weight`` / ``weight_scale`` buffers, ``load_full``,
``forward``, ``.kernel``), ``make_linear`` and ``summarize``.

Numerics follow the reference formulas exactly:

* ``quantize_rows`` (quant.py:92-100): per row ``amax = max|x|`` clamped to
  >= 1e-12, ``scale = amax / 448`` (fp8) or ``/ 127`` (int8),
  ``q = e4m3(clamp(x / scale, +-448))`` or ``int8(clamp(round(x / scale), +-127))``.
  The CUDA kernel is bit-identical to the reference (IEEE division, RNE).
* ``quantize_weight`` (quant.py:77-89): the same per output channel, scale [N].
* ``QuantLinear.forward`` (quant.py:148-197): ``y = (q_a . q_w^T) * s_a[m] * s_w[n]``
  with fp32 (e4m3) or int32 (int8) accumulation in one tcgen05 GEMM whose
  epilogue applies both scales and rounds to the layer dtype. The int32
  accumulators are bit-exact with ``torch._int_mm``; no row padding is needed
  (the reference pads to 16 / 8 rows for cuBLASLt, quant.py:167, :194).

There is no CPU path: a CPU tensor raises ``RuntimeError``. The CPU formulas
are restated in the repository's test oracle only.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn

from .. import _lib

MODES = ("auto", "none", "fp8", "int8")

_FP8 = torch.float8_e4m3fn
_FP8_MAX = 448.0
_INT8_MAX = 127.0
_EPS = 1e-12
KERNEL_NAME = "sm100a"


def _mode_code(mode: str) -> int:
    if mode == "fp8":
        return _lib.MODE_FP8
    if mode == "int8":
        return _lib.MODE_INT8
    raise ValueError(f"cannot quantize to {mode!r}")


def fp8_supported(device: Any) -> bool:
    """FP8 tensor cores present and usable by this library (reference: quant.py:37-40).

    The reference answers True from sm_89 up; the kernels here are built for sm_100a only
    (arch-specific code does not run on other compute capabilities), so only 10.0 counts."""
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(torch.device(device)) == (10, 0)


def resolve_mode(mode: str, device: Any, weight_bytes: int | None = None) -> str:
    """Turn ``auto`` into a concrete mode (reference: quant.py:43-69, same rules)."""
    if mode not in MODES:
        raise ValueError(f"unknown quant mode {mode!r}; expected one of {MODES}")
    dev = torch.device(device)
    if mode == "fp8" and dev.type == "cuda" and not fp8_supported(dev):
        major, minor = torch.cuda.get_device_capability(dev)
        raise ValueError(f"fp8 needs sm_89 or newer; this GPU is sm_{major}{minor}. Use --quant int8.")
    if mode != "auto":
        return mode
    if dev.type != "cuda":
        return "none"
    if weight_bytes:
        free, _ = torch.cuda.mem_get_info(dev)
        if free >= weight_bytes * 1.2:
            return "none"
    return "fp8" if fp8_supported(dev) else "int8"


def quantizable(in_features: int, out_features: int) -> bool:
    """Both GEMM dims divisible by 16 (reference: quant.py:72-74)."""
    return in_features % 16 == 0 and out_features % 16 == 0


def _quantize(x: torch.Tensor, mode: str) -> tuple[torch.Tensor, torch.Tensor]:
    code = _mode_code(mode)
    _lib.require_cuda(x, "quantize")
    if x.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(x.shape)}")
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        x = x.float()
    if x.stride(1) != 1 or x.stride(0) < x.shape[1]:
        x = x.contiguous()
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=_FP8 if mode == "fp8" else torch.int8, device=x.device)
    scale = torch.empty((rows,), dtype=torch.float32, device=x.device)
    if rows and cols:
        status = _lib.lib().d3b_act_quant(
            _lib.ptr(x), _lib.dtype_code(x.dtype), x.stride(0), _lib.ptr(q), _lib.ptr(scale), rows, cols, code,
            _lib.stream_of(x),
        )
        _lib.check(status, "d3b_act_quant")
    return q, scale


def quantize_weight(weight: torch.Tensor, mode: str) -> tuple[torch.Tensor, torch.Tensor]:
    """[N, K] float -> ([N, K] fp8/int8, [N] float32 per-channel scale) (quant.py:77-89)."""
    if mode not in ("fp8", "int8"):
        raise ValueError(f"cannot quantize weights to {mode!r}")
    q, scale = _quantize(weight, mode)
    return q.contiguous(), scale.contiguous()


def quantize_rows(x: torch.Tensor, mode: str) -> tuple[torch.Tensor, torch.Tensor]:
    """[M, K] activations -> (quantized [M, K], [M, 1] float32 per-token scale) (quant.py:92-100).

    The reference treats any mode other than ``fp8`` as int8; so does this.
    """
    q, scale = _quantize(x, "fp8" if mode == "fp8" else "int8")
    return q, scale[:, None]


def scaled_mm(
    q_a: torch.Tensor,
    q_w: torch.Tensor,
    scale_a: torch.Tensor | None,
    scale_w: torch.Tensor | None,
    *,
    out_dtype: torch.dtype,
) -> torch.Tensor:
    """``(q_a . q_w^T) * scale_a[m] * scale_w[n]`` -> [M, N] in ``out_dtype``.

    ``q_a`` [M, K] and ``q_w`` [N, K] are both e4m3fn or both int8 (K-major).
    ``out_dtype=torch.int32`` (int8 only) returns the raw int32 accumulators.
    """
    _lib.require_cuda(q_a, "scaled_mm")
    if q_a.dtype != q_w.dtype or q_a.dtype not in (_FP8, torch.int8):
        raise RuntimeError(f"q_a and q_w must both be float8_e4m3fn or both int8, got {q_a.dtype}, {q_w.dtype}")
    mode = _lib.MODE_FP8 if q_a.dtype == _FP8 else _lib.MODE_INT8
    if q_a.dim() != 2 or q_w.dim() != 2 or q_a.shape[1] != q_w.shape[1]:
        raise ValueError(f"shape mismatch {tuple(q_a.shape)} x {tuple(q_w.shape)}^T")
    q_a = q_a.contiguous()
    q_w = q_w.contiguous()
    rows, k = q_a.shape
    n = q_w.shape[0]
    out = torch.empty((rows, n), dtype=out_dtype, device=q_a.device)
    if rows == 0:
        return out
    sa = None if scale_a is None else scale_a.reshape(-1).float().contiguous()
    sw = None if scale_w is None else scale_w.reshape(-1).float().contiguous()
    if out_dtype != torch.int32 and (sa is None or sw is None):
        raise ValueError("scales are required unless out_dtype is torch.int32")
    status = _lib.lib().d3b_w8a8_gemm(
        _lib.ptr(q_a), _lib.ptr(q_w), _lib.ptr(sa), _lib.ptr(sw), _lib.ptr(out), n, rows, n, k, mode,
        _lib.dtype_code(out_dtype), _lib.stream_of(q_a),
    )
    _lib.check(status, "d3b_w8a8_gemm")
    return out


class QuantLinear(nn.Module):
    """A bias-free W8A8 linear (reference: quant.py:103-197), served by the sm_100a kernels."""

    def __init__(self, in_features: int, out_features: int, *, mode: str, dtype: torch.dtype, device: Any):
        super().__init__()
        if mode not in ("fp8", "int8"):
            raise ValueError(f"QuantLinear needs fp8 or int8, got {mode!r}")
        if not quantizable(in_features, out_features):
            raise ValueError(f"{out_features}x{in_features} is not a quantizable GEMM shape")
        self.in_features = in_features
        self.out_features = out_features
        self.mode = mode
        self.dtype = dtype
        self.tp_size = 1
        storage = _FP8 if mode == "fp8" else torch.int8
        self.register_buffer("weight", torch.empty(out_features, in_features, dtype=storage, device=device))
        self.register_buffer("weight_scale", torch.ones(out_features, dtype=torch.float32, device=device))
        # "sm100a" once the tcgen05 kernels have served a call; None before.
        self.kernel: str | None = None

    def extra_repr(self) -> str:
        return f"in={self.in_features}, out={self.out_features}, mode={self.mode}"

    @torch.no_grad()
    def load_full(self, full: torch.Tensor) -> None:
        if tuple(full.shape) != (self.out_features, self.in_features):
            raise ValueError(
                f"linear shape mismatch: module {(self.out_features, self.in_features)} "
                f"vs checkpoint {tuple(full.shape)}"
            )
        q, scale = quantize_weight(full.to(self.weight.device), self.mode)
        self.weight.copy_(q)
        self.weight_scale.copy_(scale)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape[:-1]
        flat = x.reshape(-1, self.in_features)
        q, scale = quantize_rows(flat, self.mode)
        out = scaled_mm(q, self.weight, scale, self.weight_scale, out_dtype=self.dtype)
        self.kernel = KERNEL_NAME
        return out.reshape(*shape, self.out_features)

    def forward_quantized(self, q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
        """The linear on input rows already quantised in this layer's mode, e.g. by the
        fused producers of ``d3_turbo_trt_b200.model.fused``: q [M, K], scale [M, 1] -> [M, N]."""
        expect = _FP8 if self.mode == "fp8" else torch.int8
        if q.dtype != expect or q.dim() != 2 or q.shape[1] != self.in_features:
            raise ValueError(f"expected [M, {self.in_features}] {expect} codes, got {tuple(q.shape)} {q.dtype}")
        out = scaled_mm(q, self.weight, scale, self.weight_scale, out_dtype=self.dtype)
        self.kernel = KERNEL_NAME
        return out


def make_linear(
    in_features: int,
    out_features: int,
    *,
    quant: str,
    dtype: torch.dtype,
    mapping: Any = None,
    tensor_parallel_mode: Any = None,
    device: Any,
) -> nn.Module:
    """:class:`QuantLinear` for fp8/int8 on a quantizable shape (reference: quant.py:214-236).

    Other projections stay dense in ``dtype`` (a bias-free ``nn.Linear``), as the
    reference keeps them in the activation dtype.
    """
    if quant in ("fp8", "int8") and quantizable(in_features, out_features):
        return QuantLinear(in_features, out_features, mode=quant, dtype=dtype, device=device)
    return nn.Linear(in_features, out_features, bias=False, dtype=dtype, device=device)


def summarize(modules: Any) -> dict[str, Any]:
    """Bytes held by quantized and unquantized linear weights, and kernels used (quant.py:239-255)."""
    quantized = dense = 0
    kernels: dict[str, int] = {}
    for module in modules:
        if isinstance(module, QuantLinear):
            quantized += module.weight.numel() * module.weight.element_size()
            key = module.kernel or "unused"
            kernels[key] = kernels.get(key, 0) + 1
        elif hasattr(module, "weight") and isinstance(getattr(module, "weight"), torch.Tensor):
            if module.weight.dim() == 2:
                dense += module.weight.numel() * module.weight.element_size()
    return {
        "quantized_gib": round(quantized / 1024**3, 3),
        "dense_linear_gib": round(dense / 1024**3, 3),
        "kernels": kernels,
    }
