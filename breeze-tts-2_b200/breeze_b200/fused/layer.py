"""FusedDecoderLayer: a transformers decoder layer's decode step on this package's kernels.

Drop-in for models/fused/layer.py: the same class name (the reference's depth
graph checks it by name, models/cudagraph/depth_decoder_graph.py:181), the
constructor ``FusedDecoderLayer(layer, layer_idx, mlp_bits=None,
attn_bits=16)`` and the decoder-layer forward signature. Calls this layer
does not handle -- no static cache with per-layer ``layers``, no rotary
embeddings or mask, or more than ``MAX_NEW_POSITIONS`` new positions -- go to
the wrapped layer unchanged.

The projections are held as one ``DecodeLayer`` (breeze_b200.fused.stack),
the same weight set the decode-step graphs launch on:

  wqkv  [q; k; v] rows, bf16 or fp8 (``attn_bits``) as a FusedWeight
  wo    the O projection, same format
  wgu   [gate; up] rows: Int4Linear tinygemm tiles or Fp8Linear codes joined
        along N as stored (no re-quantization), else a FusedWeight of
        ``mlp_bits`` (16 by default)
  wd    the down projection, in the MLP's format

A call over T new positions and B cache rows is one pass over T*B rows,
ordered position-major, so every weight is streamed once per call whatever T
is:

  qkv  = gemv(x, wqkv, RMSNorm ln1)                      one launch
  attn = attention_step(qkv rows of position t)          one launch per t; position
                                                         t sees the cache up to t
  h    = gemv(attn, wo) + x                              one launch (short caches
                                                         with bf16 O: attention, O
                                                         and + x fused, per t)
  act  = silu(g) * u, [g | u] = gemv(h, wgu, RMSNorm ln2)  one launch
  out  = gemv(act, wd) + h                               one launch
"""

from __future__ import annotations

import torch
from torch import nn

from .. import _lib
from .kernels import FusedWeight
from .stack import DecodeLayer, QWeight

MAX_NEW_POSITIONS = 4  # short prefills handled here, as the reference's layer does (layer.py:71)
# bq_attention_o_step's limits (cache length, batch rows)
_ATTN_O_MAX_S, _ATTN_O_MAX_B = 256, 4


def _join_quantized(mods) -> QWeight | None:
    """Int4Linear or Fp8Linear modules joined along N exactly as stored; None
    for plain Linears. The Int4Linear modules are re-pointed at views of the
    joined tiles, so the weight memory is not duplicated."""
    kind = type(mods[0]).__name__
    if any(type(m).__name__ != kind for m in mods):
        raise ValueError("the MLP projections mix weight formats")
    k = mods[0].in_features
    if any(m.in_features != k for m in mods):
        raise ValueError("the MLP projections differ in input width")
    if kind == "Int4Linear":
        group = mods[0].group_size
        if any(m.group_size != group for m in mods):
            raise ValueError("the MLP projections differ in int4 group size")
        tiles = torch.cat([m.weight_int4 for m in mods], 0).contiguous()
        row = 0
        for m in mods:
            n8 = m.weight_int4.shape[0]
            m.weight_int4 = tiles[row:row + n8]
            row += n8
        sz = torch.cat([m.scales_zeros for m in mods], 1).contiguous()
        return QWeight(_lib.W_INT4_TINYGEMM, tiles, sz, sum(m.out_features for m in mods), k, group)
    if kind == "Fp8Linear":
        codes = torch.cat([m.weight_fp8 for m in mods], 0).contiguous()
        scale = torch.cat([m.weight_scale.reshape(-1).float() for m in mods]).contiguous()
        return QWeight(_lib.W_FP8_E4M3, codes, scale, codes.shape[0], k)
    return None


def _packed(weights, bits: int) -> QWeight:
    return QWeight.from_fused(FusedWeight(torch.cat([w.detach() for w in weights], 0), bits))


def decode_layer_weights(layer: nn.Module, mlp_bits: int | None = None, attn_bits: int = 16) -> DecodeLayer:
    """The DecodeLayer of a transformers / Breeze decoder layer."""
    attn, mlp = layer.self_attn, layer.mlp
    qn, kn = getattr(attn, "q_norm", None), getattr(attn, "k_norm", None)
    wgu = _join_quantized([mlp.gate_proj, mlp.up_proj])
    if wgu is not None:
        wd = _join_quantized([mlp.down_proj])
    else:
        bits = mlp_bits or 16
        wgu = _packed([mlp.gate_proj.weight, mlp.up_proj.weight], bits)
        wd = _packed([mlp.down_proj.weight], bits)
    return DecodeLayer(
        wqkv=_packed([attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight], attn_bits),
        wo=_packed([attn.o_proj.weight], attn_bits), wgu=wgu, wd=wd,
        ln1=layer.input_layernorm.weight, ln2=layer.post_attention_layernorm.weight,
        q_norm=None if qn is None else qn.weight, k_norm=None if kn is None else kn.weight)


class FusedDecoderLayer(nn.Module):
    def __init__(self, layer: nn.Module, layer_idx: int, mlp_bits: int | None = None, attn_bits: int = 16):
        super().__init__()
        self.orig = layer
        self.layer_idx = layer_idx
        self.eps = float(layer.input_layernorm.variance_epsilon)
        cfg = layer.self_attn.config
        self.kv_heads = int(cfg.num_key_value_heads)
        self.head_dim = int(layer.self_attn.head_dim)
        self.weights = decode_layer_weights(layer, mlp_bits, attn_bits)

    # ---------------------------------------------------------------- dispatch
    def handles(self, hidden_states, attention_mask, past_key_values, cache_position, position_embeddings) -> bool:
        """True for a call this layer runs itself: new positions against a
        static cache, with the rotary embeddings, mask and positions given."""
        return (getattr(past_key_values, "layers", None) is not None and position_embeddings is not None
                and attention_mask is not None and cache_position is not None
                and hidden_states.shape[1] <= MAX_NEW_POSITIONS)

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                use_cache=False, cache_position=None, position_embeddings=None, **kwargs):
        if not self.handles(hidden_states, attention_mask, past_key_values, cache_position, position_embeddings):
            return self.orig(hidden_states, attention_mask=attention_mask, position_ids=position_ids,
                             past_key_values=past_key_values, use_cache=use_cache, cache_position=cache_position,
                             position_embeddings=position_embeddings, **kwargs)
        cache = past_key_values.layers[self.layer_idx]
        if not cache.is_initialized:
            blank = hidden_states.new_zeros(hidden_states.shape[0], self.kv_heads, 1, self.head_dim)
            try:
                cache.lazy_initialization(blank, blank)
            except TypeError:  # cache layers whose lazy_initialization takes the keys only
                cache.lazy_initialization(blank)
        cos, sin = position_embeddings
        out = self.step(hidden_states, cos, sin, cache_position, cache.keys, cache.values, attention_mask)
        if hasattr(cache, "cumulative_length"):
            cache.cumulative_length.add_(hidden_states.shape[1])  # the kernels wrote the new k / v
        return out

    # ---------------------------------------------------------------- compute
    def step(self, hidden_states, cos, sin, cache_position, keys, values, mask) -> torch.Tensor:
        """hidden_states (B, T, H) for cache positions ``cache_position[:T]``
        -> (B, T, H); k / v of the new positions written into ``keys`` /
        ``values`` (B, HKV, S, D)."""
        w, eps, flags = self.weights, self.eps, _lib.default_flags()
        b, t, hidden = hidden_states.shape
        rows = t * b
        x = hidden_states.transpose(0, 1).reshape(rows, hidden)  # position-major rows
        qkv = _lib.gemv(x, w.wqkv.w, w.wqkv.wfmt, w.wqkv.N, scale=w.wqkv.scale, group=w.wqkv.group, gamma=w.ln1,
                        eps=eps, flags=flags)
        fuse_o = (w.wo.wfmt == _lib.W_BF16 and x.dtype == torch.bfloat16 and keys.shape[2] <= _ATTN_O_MAX_S
                  and b <= _ATTN_O_MAX_B)
        if fuse_o:
            h = torch.empty(rows, w.wo.N, device=x.device, dtype=x.dtype)
        else:
            attn = torch.empty(rows, w.wo.K, device=x.device, dtype=torch.bfloat16)
        for p in range(t):
            sel = slice(p * b, (p + 1) * b)
            args = (qkv[sel], cos[:, p:p + 1], sin[:, p:p + 1], cache_position[p:p + 1], keys, values)
            if fuse_o:
                _lib.attention_o_step(*args, w.q_norm, w.k_norm, eps, w.wo.w, x[sel], out=h[sel], flags=flags,
                                      mask=mask[:, :, p:p + 1])
            else:
                _lib.attention_step(*args, mask[:, :, p:p + 1], w.q_norm, w.k_norm, eps, out=attn[sel], flags=flags)
        if not fuse_o:
            h = _lib.gemv(attn, w.wo.w, w.wo.wfmt, w.wo.N, scale=w.wo.scale, group=w.wo.group,
                          epilogue=_lib.EPI_ADD_RESIDUAL, residual=x, flags=flags)
        act = _lib.gemv(h, w.wgu.w, w.wgu.wfmt, w.wgu.N, scale=w.wgu.scale, group=w.wgu.group, gamma=w.ln2, eps=eps,
                        epilogue=_lib.EPI_SILU_MUL, flags=flags)
        out = _lib.gemv(act, w.wd.w, w.wd.wfmt, w.wd.N, scale=w.wd.scale, group=w.wd.group,
                        epilogue=_lib.EPI_ADD_RESIDUAL, residual=h, flags=flags)
        return out.reshape(t, b, hidden).transpose(0, 1).contiguous()

    def warm_up(self, batch_size: int, max_cache_len: int, positions: int = 1) -> None:
        """A step of ``positions`` new positions on scratch caches at this
        batch size and cache length, outside any graph capture: sizes the
        shared workspaces (they may not grow during a capture). Positions
        0.., identity rotary embedding, zero inputs."""
        dev, dtype, hidden = self.weights.ln1.device, torch.bfloat16, self.weights.wqkv.K
        keys = torch.zeros(batch_size, self.kv_heads, max_cache_len, self.head_dim, device=dev, dtype=dtype)
        values = torch.zeros_like(keys)
        cos = torch.ones(batch_size, positions, self.head_dim, device=dev, dtype=dtype)
        sin = torch.zeros_like(cos)
        mask = torch.zeros(batch_size, 1, positions, max_cache_len, device=dev, dtype=dtype)
        x = torch.zeros(batch_size, positions, hidden, device=dev, dtype=dtype)
        with torch.no_grad():
            self.step(x, cos, sin, torch.arange(positions, dtype=torch.int64, device=dev), keys, values, mask)
