"""Fused decode-step forward for a decoder layer, on this package's kernels.

Same class, constructor and forward contract as the reference's
models/fused/layer.py (FusedDecoderLayer(layer, layer_idx, mlp_bits=None,
attn_bits=16), :32-99): calls that are not a single-token decode step against
a static cache go to the wrapped layer; a short prefill (T <= 4, the depth
decoder's 2-position start) runs as T decode steps; a decode step is

    qkv = rms_gemv(x, Wqkv, ln1)                  bq_gemv, RMSNorm fused
    attn = attention_step(qkv, cos, sin, pos, k_cache, v_cache, mask, q_norm, k_norm)
    h = gemv(attn, Wo) + x                        residual epilogue
    act = silu(gate) * up = gemv(norm(h), Wgu)    RMSNorm and SiLU*up fused
    out = gemv(act, Wd) + h                       residual epilogue

Where the reference keeps tinygemm matmuls for an Int4Linear MLP with separate
rmsnorm / silu_mul / add kernels around them (:92-96), here the int4 gate and
up codes are one tinygemm tensor read by a single SiLU-epilogue launch: the
layer concatenates them once and points the modules' own ``weight_int4``
buffers at the two halves, so no weight memory is duplicated.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _lib
from .kernels import FusedWeight, attention_step, rms_gemv
from .stack import QWeight


def _from_fp8(*mods) -> FusedWeight:
    """Fp8Linear buffers (e4m3 (N, K), per-row scale (1, N)) concatenated along N."""
    w = torch.cat([m.weight_fp8 for m in mods], 0).contiguous()
    s = torch.cat([m.weight_scale.reshape(-1) for m in mods], 0).float().contiguous()
    return FusedWeight.from_parts(8, w, s)


def _fuse_int4_gate_up(gate, up) -> QWeight:
    if gate.group_size != up.group_size or gate.in_features != up.in_features:
        raise ValueError("gate and up projections differ in group size or input width")
    n8 = gate.weight_int4.shape[0]
    w = torch.cat([gate.weight_int4, up.weight_int4], 0).contiguous()
    gate.weight_int4 = w[:n8]
    up.weight_int4 = w[n8:]
    sz = torch.cat([gate.scales_zeros, up.scales_zeros], 1).contiguous()
    return QWeight(_lib.W_INT4_TINYGEMM, w, sz, 2 * gate.out_features, gate.in_features, gate.group_size)


class FusedDecoderLayer(nn.Module):
    def __init__(self, layer: nn.Module, layer_idx: int, mlp_bits: int | None = None, attn_bits: int = 16):
        super().__init__()
        self.orig = layer
        self.layer_idx = layer_idx
        attn = layer.self_attn
        self.eps = float(layer.input_layernorm.variance_epsilon)
        self.hkv = int(attn.config.num_key_value_heads)
        self.hd = int(attn.head_dim)
        self.ln1 = layer.input_layernorm.weight
        self.ln2 = layer.post_attention_layernorm.weight
        qn, kn = getattr(attn, "q_norm", None), getattr(attn, "k_norm", None)
        self.qn = qn.weight if qn is not None else None
        self.kn = kn.weight if kn is not None else None
        wq, wk, wv = attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight
        self.wqkv = FusedWeight(torch.cat([wq, wk, wv], 0).detach(), attn_bits)
        self.wo = FusedWeight(attn.o_proj.weight.detach(), attn_bits)
        mlp = layer.mlp
        kind = type(mlp.gate_proj).__name__
        self.wgu = self.wd = None
        self.qgu = self.qd = None
        if kind == "Int4Linear":
            self.qgu = _fuse_int4_gate_up(mlp.gate_proj, mlp.up_proj)
            self.qd = QWeight.from_module(mlp.down_proj)
        elif kind == "Fp8Linear":
            self.wgu = _from_fp8(mlp.gate_proj, mlp.up_proj)
            self.wd = _from_fp8(mlp.down_proj)
        else:
            bits = mlp_bits or 16
            self.wgu = FusedWeight(torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight], 0).detach(), bits)
            self.wd = FusedWeight(mlp.down_proj.weight.detach(), bits)

    def _gemv(self, x, qw: QWeight, gamma=None, epilogue=_lib.EPI_NONE, residual=None):
        return _lib.gemv(x, qw.w, qw.wfmt, qw.N, scale=qw.scale, group=qw.group, gamma=gamma, eps=self.eps,
                         epilogue=epilogue, residual=residual, flags=_lib.default_flags())

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                use_cache=False, cache_position=None, position_embeddings=None, **kwargs):
        layers = getattr(past_key_values, "layers", None)
        T = hidden_states.shape[1]
        if layers is None or position_embeddings is None or attention_mask is None or cache_position is None or T > 4:
            return self.orig(hidden_states, attention_mask=attention_mask, position_ids=position_ids,
                             past_key_values=past_key_values, use_cache=use_cache, cache_position=cache_position,
                             position_embeddings=position_embeddings, **kwargs)
        if T > 1:
            # a short prefill is exactly T causal decode steps: same rope, mask rows and cache
            cos, sin = position_embeddings
            outs = []
            for t in range(T):
                outs.append(self.forward(
                    hidden_states[:, t:t + 1], attention_mask=attention_mask[:, :, t:t + 1],
                    position_ids=None if position_ids is None else position_ids[:, t:t + 1],
                    past_key_values=past_key_values, use_cache=use_cache, cache_position=cache_position[t:t + 1],
                    position_embeddings=(cos[:, t:t + 1], sin[:, t:t + 1])))
            return torch.cat(outs, dim=1)
        cache = layers[self.layer_idx]
        if not cache.is_initialized:
            z = hidden_states.new_zeros(hidden_states.shape[0], self.hkv, 1, self.hd)
            try:
                cache.lazy_initialization(z, z)
            except TypeError:  # caches whose lazy_initialization takes the keys only
                cache.lazy_initialization(z)
        x = hidden_states[:, 0]
        qkv = rms_gemv(x, self.wqkv, self.ln1, self.eps)
        cos, sin = position_embeddings
        if self.wo.bits == 16 and x.dtype == torch.bfloat16 and cache.keys.shape[2] <= 256 and x.shape[0] <= 4:
            # short cache (the depth decoder): attention, O projection and residual in one launch
            h = _lib.attention_o_step(qkv, cos, sin, cache_position, cache.keys, cache.values, self.qn, self.kn,
                                      self.eps, self.wo.w, x, flags=_lib.default_flags(), mask=attention_mask)
        else:
            attn = attention_step(qkv, cos, sin, cache_position, cache.keys, cache.values, attention_mask, self.qn,
                                  self.kn, self.eps)
            h = rms_gemv(attn, self.wo, None, epilogue=_lib.EPI_ADD_RESIDUAL, residual=x)
        if hasattr(cache, "cumulative_length"):
            cache.cumulative_length.add_(1)  # the kernel wrote the new k / v; keep the cache's own count
        if self.qgu is not None:
            act = self._gemv(h, self.qgu, gamma=self.ln2, epilogue=_lib.EPI_SILU_MUL)
            out = self._gemv(act, self.qd, epilogue=_lib.EPI_ADD_RESIDUAL, residual=h)
        else:
            act = rms_gemv(h, self.wgu, self.ln2, self.eps, epilogue=_lib.EPI_SILU_MUL)
            out = rms_gemv(act, self.wd, None, epilogue=_lib.EPI_ADD_RESIDUAL, residual=h)
        return out.unsqueeze(1)
