"""The d3 backbone's state-once prefill on the sm_100a kernels (config 4 end to end).

``D3Backbone`` runs the reference's ``D3Core`` schedule (d3trt/model/core.py:146-181):
the state block once through every layer, keeping one snapshot entry per layer
(``AttentionEntry`` keys/values, ``DeltaEntry`` conv tail and recurrent state,
core.py:28-40), then the question blocks through every layer against that
snapshot, and the final norm of each block's last real token. The layer math is
core.py:193-402 (``_layer``, ``_attention``, ``_delta``) with the model's modules
(transformers' Qwen3.5: zero-centred RMSNorm, gated attention, Gated DeltaNet, SiLU
MLP). Where the reference calls a module, this file calls a kernel of this
library:

* input_layernorm / post_attention_layernorm + the residual add, fused with the
  per-row FP8/INT8 quantisation of the rows every projection of the layer reads
  (``fused.add_rmsnorm_quant``); one set of codes feeds q/k/v_proj (or the four
  GDN input projections, or gate/up_proj);
* every Linear: ``QuantLinear`` (W8A8, tcgen05 GEMM, dequant fused);
* attention: ``state_attention`` for the state pass, ``prefix_bidir_attention``
  for the question pass, then ``out * sigmoid(gate)`` fused with o_proj's
  quantisation (``fused.sigmoid_gate_quant``);
* the GDN layers' causal convolution + SiLU: ``conv.causal_conv1d_silu`` on the
  in_proj output as the GEMM writes it (token-major; reads the snapshot's tail in
  place of the reference's concatenation), its q/k/v handed on as strided views;
* the GDN scan of the question pass: ``gdn.question_gated_delta_rule`` (one
  shared initial state, no per-row copy or head repeat); of the state pass:
  ``gdn.chunk_gated_delta_rule`` (64-token chunks with the inter-chunk state
  recurrence on the tensor cores), or FLA's chunked kernel when the caller selects
  it (``gdn_state="fla"``: the reference's own GPU path for that call);
* SiLU(gate) * up fused with down_proj's quantisation (``fused.silu_mul_quant``) and
  the GDN output's gated RMSNorm fused with out_proj's (``fused.gated_rmsnorm_quant``);
* the 255-way readout: ``readout.probabilities_tensor``.

The rest stays on the reference's own formulas in torch: q/k RMSNorm and the
rotary embedding (transformers' ``apply_rotary_pos_emb``) of the 16 attention
layers, and the GDN gates g and beta. ``causal_conv1d``, ``gated_rms_norm`` below
are the reference's torch forms, kept as the checks of the kernels.
Weights are taken by the model's own parameter names (``layers.{i}.self_attn.
q_proj.weight``, ...), so a checkpoint or a transformers model's ``state_dict``
loads as it is.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Mapping, Sequence

import torch
import torch.nn.functional as F

from ..kernels import prefix_bidir as pb
from . import fused, gdn
from .conv import causal_conv1d_silu
from .quant import QuantLinear, quantizable, quantize_rows
from .readout import probabilities_tensor
from .snapshot import AttentionEntry, DeltaEntry

Snapshot = list


@dataclass
class BackboneConfig:
    """The text model's shape (transformers Qwen3_5TextConfig field names)."""

    hidden_size: int = 5120
    intermediate_size: int = 17408
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 48
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000_000.0
    partial_rotary_factor: float = 0.25
    layer_types: list = field(default_factory=lambda: (["linear_attention"] * 3 + ["full_attention"]) * 16)

    @property
    def key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim


def rotary_tables(config: BackboneConfig, positions: torch.Tensor, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) [B, T, rotary_dim] for integer positions [B, T]: the default RoPE of
    Qwen3_5TextRotaryEmbedding over head_dim * partial_rotary_factor dimensions, in fp32,
    cast to ``dtype``. Text positions are the same on its three M-RoPE axes, so the
    interleaving of the axes changes nothing."""
    dim = int(config.head_dim * config.partial_rotary_factor)
    inv_freq = 1.0 / (config.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64, device=positions.device)
                                            .float() / dim))
    freqs = positions.float()[..., None] * inv_freq  # [B, T, dim/2]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rotary(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """transformers' apply_rotary_pos_emb (partial rotary): q/k [B, H, T, D], cos/sin [B, T, r]."""
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    r = cos.shape[-1]

    def rot(x):
        xr, xp = x[..., :r], x[..., r:]
        x1, x2 = xr[..., : r // 2], xr[..., r // 2:]
        return torch.cat([(xr * cos) + (torch.cat((-x2, x1), dim=-1) * sin), xp], dim=-1)

    return rot(q), rot(k)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3_5RMSNorm: fp32 normalisation, times (1 + w) in fp32, back to x's dtype."""
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (out * (1.0 + weight.float())).type_as(x)


def gated_rms_norm(x: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3_5RMSNormGated: normalise in fp32, times w in x's dtype, times silu(gate) in fp32."""
    dtype = x.dtype
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = weight * xf.to(dtype)
    return (y * F.silu(gate.float())).to(dtype)


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Causal depthwise convolution over [B, C, L] with SiLU (ops.py:266-285, the torch form)."""
    out = F.conv1d(x, weight.unsqueeze(1), None, padding=weight.shape[-1] - 1, groups=x.shape[1])
    return F.silu(out[..., : x.shape[-1]])


class _Linear:
    """A projection: QuantLinear where the shape is quantizable (quant.py:72-74), else bf16."""

    def __init__(self, weight: torch.Tensor, mode: str, device: torch.device):
        n, k = weight.shape
        self.quant = quantizable(k, n)
        if self.quant:
            self.mod = QuantLinear(k, n, mode=mode, dtype=torch.bfloat16, device=device)
            self.mod.load_full(weight.to(device=device, dtype=torch.bfloat16))
        else:
            self.weight = weight.to(device=device, dtype=torch.bfloat16)
        self.mode = mode

    def from_codes(self, codes: torch.Tensor, scale: torch.Tensor, rows: torch.Tensor | None) -> torch.Tensor:
        """The projection of rows already quantised in this layer's mode (``rows``: the bf16
        rows themselves, for a projection kept in bf16; None where the shape is quantizable)."""
        if self.quant:
            return self.mod.forward_quantized(codes, scale)
        if rows is None:
            raise ValueError("a projection fed by the fused norm's codes must have a quantizable shape")
        return F.linear(rows, self.weight)

    def __call__(self, x2d: torch.Tensor) -> torch.Tensor:
        if self.quant:
            return self.mod(x2d)
        return F.linear(x2d, self.weight)


class D3Backbone:
    """State-once prefill of the d3 text backbone on this library's kernels (see the module doc)."""

    def __init__(self, config: BackboneConfig, weights: Mapping[str, torch.Tensor], *, device: torch.device,
                 mode: str = "fp8", gdn_state: str = "ours"):
        if gdn_state not in ("ours", "fla"):
            raise ValueError("gdn_state is 'ours' or 'fla'")
        self.config, self.device, self.mode, self.gdn_state = config, torch.device(device), mode, gdn_state
        c = config
        dev = self.device

        def w(name: str) -> torch.Tensor:
            return weights[name].to(device=dev)

        self.embed = w("embed_tokens.weight").to(torch.bfloat16)
        self.final_norm = w("norm.weight")
        self.layers = []
        for i, kind in enumerate(c.layer_types):
            p = f"layers.{i}."
            L = {"kind": kind, "in_w1": 1.0 + w(p + "input_layernorm.weight").float(),
                 "post_w1": 1.0 + w(p + "post_attention_layernorm.weight").float()}
            gate_up = torch.cat([w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight")], 0)
            L["gate_up"] = _Linear(gate_up, mode, dev)
            L["down"] = _Linear(w(p + "mlp.down_proj.weight"), mode, dev)
            if kind == "full_attention":
                a = p + "self_attn."
                for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
                    L[n] = _Linear(w(a + n + ".weight"), mode, dev)
                L["q_norm"], L["k_norm"] = w(a + "q_norm.weight"), w(a + "k_norm.weight")
            elif kind == "linear_attention":
                a = p + "linear_attn."
                # the four input projections read the same codes: one GEMM over their rows
                # stacked (per-output-channel scales, so every output equals the separate
                # projection's), sliced afterwards into qkv, z, b and a
                parts = [w(a + n + ".weight") for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")]
                L["in_proj"] = _Linear(torch.cat(parts, 0), mode, dev)
                L["in_split"] = tuple(int(t.shape[0]) for t in parts)
                del parts
                L["out_proj"] = _Linear(w(a + "out_proj.weight"), mode, dev)
                L["conv"] = w(a + "conv1d.weight").squeeze(1)
                L["A_log"], L["dt_bias"], L["norm"] = w(a + "A_log"), w(a + "dt_bias"), w(a + "norm.weight")
                L["neg_exp_a"] = -L["A_log"].float().exp()  # the gates' per-head constants, formed once
                L["dt_bias_f"] = L["dt_bias"].float()
            else:
                raise ValueError(f"unknown layer type {kind!r}")
            fed = ("q_proj", "k_proj", "v_proj", "o_proj", "in_proj", "out_proj", "gate_up", "down")
            for n in fed:
                if n in L and not L[n].quant:
                    raise ValueError(f"layer {i} {n}: every projection reads fused-producer codes and must be "
                                     "quantizable (in and out features divisible by 16)")
            self.layers.append(L)

    # ------------------------------------------------------------------
    def embed_ids(self, ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(ids.to(self.device), self.embed)

    def state(self, ids: torch.Tensor) -> Snapshot:
        """``ids`` [1, S] -> snapshot (one entry per layer), as core.py:146-156."""
        embeds = self.embed_ids(ids)
        positions = torch.arange(ids.shape[1], device=self.device)[None]
        rope = rotary_tables(self.config, positions, embeds.dtype)
        snapshot: Snapshot = []
        hidden, delta = embeds, None
        for L in self.layers:
            hidden, delta, entry = self._layer(L, hidden, delta, rope, None, None, None)
            snapshot.append(entry)
        return snapshot

    def questions(self, snapshot: Snapshot, ids: torch.Tensor, lengths: Sequence[int], *,
                  state_len: int) -> torch.Tensor:
        """``ids`` [B, W] right-padded -> final-norm hidden [B, hidden] at each block's last
        token, as core.py:158-181 (padding rows zeroed at the embedding)."""
        rows, width = ids.shape
        lengths = [int(n) for n in lengths]
        lens_t = torch.tensor(lengths, device=self.device)
        present = torch.arange(width, device=self.device)[None, :] < lens_t[:, None]
        embeds = self.embed_ids(ids) * present[..., None].to(torch.bfloat16)
        positions = (state_len + torch.arange(width, device=self.device))[None].expand(rows, -1)
        rope = rotary_tables(self.config, positions, embeds.dtype)
        lens_d = lens_t.to(torch.int32)
        hidden, delta = embeds, None
        for L, entry in zip(self.layers, snapshot):
            hidden, delta, _ = self._layer(L, hidden, delta, rope, entry, lengths, lens_d)
        hidden = hidden + delta  # the last layer's residual add
        last = hidden[torch.arange(rows, device=self.device), lens_t - 1]
        return rms_norm(last, self.final_norm, self.config.rms_norm_eps)

    def probabilities(self, hidden: torch.Tensor, readout: torch.Tensor, counts, *, temperature: float = 1.0):
        """[B, n_opt] fp32 probabilities (trtllm_stack.py:451-468) on the device."""
        return probabilities_tensor(hidden, readout, counts, temperature=temperature)

    # ------------------------------------------------------------------
    def _layer(self, L, hidden, delta, rope, entry, lengths, lens_d):
        """One decoder layer (core.py:193-226). ``hidden`` + ``delta`` is the layer input (the
        previous layer's MLP output not yet added); returns (hidden, mlp output, entry) so the
        next layer's residual add is fused with its norm."""
        c = self.config
        rows, T, H = hidden.shape
        res, q, s = fused.add_rmsnorm_quant(hidden, delta, L["in_w1"], c.rms_norm_eps, self.mode)
        if L["kind"] == "full_attention":
            mixed, entry = self._attention(L, q, s, rows, T, rope, entry, lengths, lens_d)
        else:
            mixed, entry = self._delta(L, q, s, rows, T, entry)
        h2, q2, s2 = fused.add_rmsnorm_quant(res, mixed.view(rows, T, H), L["post_w1"], c.rms_norm_eps, self.mode)
        gu = L["gate_up"].from_codes(q2, s2, None)  # [M, 2I]: gate, then up
        qa, sa = fused.silu_mul_quant(gu, self.mode)  # silu(gate_proj(x)) * up_proj(x), quantised for down_proj
        down = L["down"].from_codes(qa, sa, None).view(rows, T, H)
        return h2, down, entry

    def _attention(self, L, q, s, rows, T, rope, entry, lengths, lens_d):
        """core.py:228-297: gated attention; the state pass keeps K/V, the question pass reads them."""
        c = self.config
        D, Hq, Hkv = c.head_dim, c.num_attention_heads, c.num_key_value_heads
        qg = L["q_proj"].from_codes(q, s, None).view(rows, T, Hq, 2 * D)
        gate = qg[..., D:]
        cos, sin = rope
        # q_norm / k_norm and the partial rotary embedding in one kernel each, written
        # token-major [rows, T, heads, D]; the attention reads [rows, heads, T, D] views
        query = fused.qk_norm_rope(qg[..., :D], L["q_norm"], cos, sin, c.rms_norm_eps).transpose(1, 2)
        key = fused.qk_norm_rope(L["k_proj"].from_codes(q, s, None).view(rows, T, Hkv, D), L["k_norm"], cos, sin,
                                 c.rms_norm_eps).transpose(1, 2)
        # the kernels read K and V through one set of strides: v_proj's output is already
        # token-major like K, so V is a view of it
        value = L["v_proj"].from_codes(q, s, None).view(rows, T, Hkv, D).transpose(1, 2)
        scale = D ** -0.5
        if entry is None:
            out = pb.state_attention(query, key, value, scale=scale)
            entry = AttentionEntry(keys=key, values=value)
        else:
            out = pb.prefix_bidir_attention(query, entry.keys[0], entry.values[0], key, value, lens_d, scale=scale)
        qo, so = fused.sigmoid_gate_quant(out.transpose(1, 2), gate, self.mode)
        return L["o_proj"].from_codes(qo, so, None), entry

    def _delta(self, L, q, s, rows, T, entry):
        """core.py:299-402: Gated DeltaNet mixer."""
        c = self.config
        window = c.linear_conv_kernel_dim - 1
        HV, HK, Dk, Dv = c.linear_num_value_heads, c.linear_num_key_heads, c.linear_key_head_dim, c.linear_value_head_dim
        proj = L["in_proj"].from_codes(q, s, None)  # [rows * T, qkv | z | b | a]
        nq, nz, nb, _ = L["in_split"]
        mixed = proj[:, :nq].view(rows, T, nq)  # token-major [rows, T, conv_dim], rows of the fused width
        z = proj[:, nq:nq + nz].view(rows, T, HV, Dv)
        b, a = proj[:, nq + nz:nq + nz + nb], proj[:, nq + nz + nb:]
        if entry is None:
            conv = causal_conv1d_silu(mixed, L["conv"])
            # [1, conv_dim, window], as core.py:321; copied so the snapshot does not hold the projection
            tail = mixed[:, -window:, :].transpose(1, 2).contiguous()
            if tail.shape[-1] < window:
                tail = F.pad(tail, (window - tail.shape[-1], 0))
            initial = None
        else:
            tail, initial = entry.tail, entry.recurrent
            conv = causal_conv1d_silu(mixed, L["conv"], tail)  # reads the tail in place: no cat
            initial = initial.expand(rows, -1, -1, -1)
        kd = c.key_dim
        query = conv[..., :kd].view(rows, T, HK, Dk)  # strided views: the scan reads them in place
        key = conv[..., kd:2 * kd].view(rows, T, HK, Dk)
        value = conv[..., 2 * kd:].view(rows, T, HV, Dv)
        g, beta = fused.gdn_gates(a, b, L["neg_exp_a"], L["dt_bias_f"])  # core.py:341-342 in one kernel
        g, beta = g.view(rows, T, HV), beta.view(rows, T, HV)
        if entry is None:
            core, final = self._state_scan(query, key, value, g, beta)
            entry = DeltaEntry(tail=tail, recurrent=final)
        else:
            core, _ = gdn.question_gated_delta_rule(query, key, value, g=g, beta=beta, initial_state=initial,
                                                    output_final_state=False, use_qk_l2norm_in_kernel=True)
        qo, so = fused.gated_rmsnorm_quant(core.reshape(rows * T, -1), z.reshape(rows * T, -1), L["norm"],
                                           c.rms_norm_eps, Dv, self.mode)  # Qwen3_5RMSNormGated, then out_proj's codes
        return L["out_proj"].from_codes(qo, so, None), entry

    def _state_scan(self, query, key, value, g, beta):
        if self.gdn_state == "fla":
            from fla.ops.gated_delta_rule import chunk_gated_delta_rule

            rep = value.shape[2] // query.shape[2]
            return chunk_gated_delta_rule(query.repeat_interleave(rep, 2), key.repeat_interleave(rep, 2),
                                          value.contiguous(),
                                          g=g, beta=beta, initial_state=None, output_final_state=True,
                                          use_qk_l2norm_in_kernel=True)
        return gdn.gated_delta_rule(query, key, value, g=g, beta=beta, initial_state=None, output_final_state=True,
                                    use_qk_l2norm_in_kernel=True, algo="chunk_state")
