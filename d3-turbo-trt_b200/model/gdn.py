"""Gated delta rule (the GDN layers' scan) on sm_100a: drop-ins for the reference's
``ops.recurrent_gated_delta_rule`` and ``ops.chunk_gated_delta_rule``
(d3trt/model/ops.py:287-360), which D3Core calls per GDN layer (core.py:348-372).

All names run ``d3b_gated_delta_rule`` (``csrc/gated_delta.cu``): ``recurrent_...`` the
token-recurrent form with an fp32 state (the math of FLA's fused recurrent kernel, the
reference's path for question blocks); ``chunk_...`` and ``question_...`` the chunked (WY)
form on the tensor cores for blocks of <= 64 tokens sharing one initial state, falling back
to the recurrence elsewhere (for the 4096-token state pass that is slower than FLA's chunked
kernel). Differences from the reference's call, all optional for the caller:

* q/k may keep H < HV heads (value head hv reads q/k head hv // (HV // H)), so the
  ``repeat_interleave`` of core.py:345-347 can be dropped;
* ``initial_state`` may be a stride-0 expand of one ``[1, HV, K, V]`` state, so the
  question pass needs no per-row copy of the snapshot's state (core.py:331).

There is no CPU path: CPU tensors raise.
"""

from __future__ import annotations

import torch

from .. import _lib


_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Per-device scratch for the chunked form's state tiles, grown on demand and reused; the
    calls that use it are ordered on the stream."""
    if nbytes == 0:
        return None
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, torch.cuda.current_stream(index).cuda_stream)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = buf
    return buf


def _strides3(t: torch.Tensor, what: str) -> object:
    if t.stride(-1) != 1:
        raise RuntimeError(f"{what}: the last dimension must be contiguous")
    return _lib.i64_array(t.stride()[:3])


ALGOS = {"auto": 0, "recurrent": 1, "chunk": 2, "chunk_state": 3}


def gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, g: torch.Tensor, beta: torch.Tensor,
                     initial_state: torch.Tensor | None = None, output_final_state: bool = False,
                     use_qk_l2norm_in_kernel: bool = True, scale: float | None = None,
                     out: torch.Tensor | None = None, algo: str = "auto") -> tuple[torch.Tensor, torch.Tensor | None]:
    """(o [B,T,HV,V] in v's dtype, final state [B,HV,K,V] fp32 or None).

    ``algo``: "recurrent" (token recurrence, fp32 throughout), "chunk" (the chunked form on
    the tensor cores: blocks of <= 64 tokens, K = V = 128, one initial state for all rows,
    no final state), "chunk_state" (64-token chunks carried through an inter-chunk state
    recurrence on the tensor cores: any length, K = V = 128, final state; FLA's
    chunk_gated_delta_rule numerics) or "auto" ("chunk" where it applies, else
    "chunk_state" where it applies, else "recurrent").
    """
    if algo not in ALGOS:
        raise ValueError(f"algo must be one of {sorted(ALGOS)}, got {algo!r}")
    for t, name in ((q, "q"), (k, "k"), (v, "v"), (g, "g"), (beta, "beta")):
        _lib.require_cuda(t, f"gated_delta_rule {name}")
    if q.dim() != 4 or k.shape != q.shape or v.dim() != 4:
        raise RuntimeError(f"gated_delta_rule: q, k [B,T,H,K] and v [B,T,HV,V] expected, got {tuple(q.shape)}, "
                           f"{tuple(k.shape)}, {tuple(v.shape)}")
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if v.shape[:2] != (B, T) or HV % H != 0:
        raise RuntimeError("gated_delta_rule: v must be [B,T,HV,V] with HV a multiple of q/k's heads")
    if q.dtype not in (torch.bfloat16, torch.float16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise RuntimeError(f"gated_delta_rule: q, k, v must share fp16/bf16, got {q.dtype}, {k.dtype}, {v.dtype}")
    if g.shape != (B, T, HV) or beta.shape != (B, T, HV):
        raise RuntimeError(f"gated_delta_rule: g and beta must be [B,T,HV] = {(B, T, HV)}")
    if K not in (64, 128) or V % 32 != 0:
        raise RuntimeError(f"gated_delta_rule: head dims K in (64, 128) and V % 32 == 0 supported, got {K}, {V}")
    e = K // 32  # the kernel copies q/k rows e elements (2e bytes) per lane
    if q.stride(-1) != 1 or q.data_ptr() % (2 * e) or any(st % e for st in q.stride()[:3]):
        q = q.contiguous() if q.stride(-1) != 1 or any(st % e for st in q.stride()[:3]) else q.clone()
    if k.stride(-1) != 1 or k.data_ptr() % (2 * e) or any(st % e for st in k.stride()[:3]):
        k = k.contiguous() if k.stride(-1) != 1 or any(st % e for st in k.stride()[:3]) else k.clone()
    if v.stride(-1) != 1:
        v = v.contiguous()
    g = g.float()
    if beta.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        beta = beta.float()
    h0, h0s = None, None
    if initial_state is not None:
        h0 = initial_state.float()
        if h0.dim() == 3:
            h0 = h0.unsqueeze(0)
        h0 = h0.expand(B, HV, K, V)
        if h0.stride(-1) != 1:
            h0 = h0.contiguous()
        h0s = _lib.i64_array(h0.stride()[:3])
    if out is None:
        out = torch.empty(B, T, HV, V, dtype=v.dtype, device=v.device)
    elif out.shape != (B, T, HV, V) or out.dtype != v.dtype or out.stride(-1) != 1:
        raise RuntimeError("gated_delta_rule: out must be [B,T,HV,V] in v's dtype with a contiguous last dim")
    ht = torch.empty(B, HV, K, V, dtype=torch.float32, device=v.device) if output_final_state else None
    question_form = (K == 128 and V == 128 and T <= 64 and not output_final_state
                     and (h0 is None or h0.stride(0) == 0 or B == 1))
    if algo == "recurrent":
        ws = None
    elif algo == "chunk" or (algo == "auto" and question_form):
        ws = _workspace(v.device, int(_lib.lib().d3b_gated_delta_workspace_size(HV, K, V)))
    else:  # the inter-chunk form: every chunk's operand tiles
        ws = _workspace(v.device, int(_lib.lib().d3b_gated_delta_state_workspace_size(B, T, HV, K, V)))
    with torch.cuda.device(v.device):
        st = _lib.lib().d3b_gated_delta_rule(
            _lib.ptr(q), _strides3(q, "q"), _lib.ptr(k), _strides3(k, "k"), _lib.ptr(v), _strides3(v, "v"),
            _lib.ptr(g), _lib.i64_array(g.stride()), _lib.ptr(beta), _lib.dtype_code(beta.dtype),
            _lib.i64_array(beta.stride()), _lib.ptr(h0), h0s, _lib.ptr(out), _strides3(out, "out"), _lib.ptr(ht),
            B, T, H, HV, K, V, _lib.dtype_code(v.dtype), float(K ** -0.5 if scale is None else scale),
            1 if use_qk_l2norm_in_kernel else 0, ALGOS[algo], _lib.ptr(ws), 0 if ws is None else ws.numel(),
            _lib.stream_of(v))
    _lib.check(st, "d3b_gated_delta_rule")
    return out, ht


def recurrent_gated_delta_rule(q, k, v, *, g, beta, initial_state, output_final_state,
                               use_qk_l2norm_in_kernel=True):
    """Drop-in for d3trt/model/ops.py:327-360 (FLA fused_recurrent_gated_delta_rule): the token recurrence."""
    return gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=initial_state,
                            output_final_state=output_final_state, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
                            algo="recurrent")


def chunk_gated_delta_rule(q, k, v, *, g, beta, initial_state, output_final_state, use_qk_l2norm_in_kernel=True):
    """Drop-in for d3trt/model/ops.py:287-324 (FLA chunk_gated_delta_rule): on the tensor cores, the
    question blocks' chunked form where it applies (blocks of <= 64 tokens sharing one state, no final
    state), else 64-token chunks with the inter-chunk state recurrence (the state pass)."""
    return gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=initial_state,
                            output_final_state=output_final_state, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)


def question_gated_delta_rule(q, k, v, *, g, beta, initial_state, output_final_state,
                              use_qk_l2norm_in_kernel=True):
    """For the question pass, with ``recurrent_gated_delta_rule``'s arguments (the call core.py:360-372
    makes for blocks of <= 256 tokens): the chunked form on the tensor cores where it applies, else the
    token recurrence."""
    return gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=initial_state,
                            output_final_state=output_final_state, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
