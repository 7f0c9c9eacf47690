"""Install fused decode layers on a model's backbone and depth decoder.

Same functions and signatures as the reference's models/fused/install.py
(install_fused_backbone :16-39, install_fused_depth :42-65): every decoder
layer is wrapped in this package's FusedDecoderLayer, then each layer runs one
decode step on a scratch static cache outside any graph capture. Nothing is
tuned here (the kernels need no autotuning); the step sizes the per-device
workspaces, which may not grow during capture.
"""

from __future__ import annotations

import torch

from .layer import FusedDecoderLayer


def _static_cache(config, max_cache_len: int, batch_size: int):
    from transformers import StaticCache

    try:
        return StaticCache(config=config, max_cache_len=max_cache_len, batch_size=batch_size)
    except TypeError:  # caches sized by their first update
        return StaticCache(config=config, max_cache_len=max_cache_len)


def _warm(stack, batch_size: int, max_seq: int) -> None:
    dev = next(stack.parameters()).device
    dtype = next(stack.parameters()).dtype
    cache = _static_cache(stack.config, max_seq, batch_size)
    x = torch.zeros(batch_size, 1, stack.config.hidden_size, device=dev, dtype=dtype)
    mask = torch.zeros(batch_size, 1, 1, max_seq, device=dev, dtype=dtype)
    pos = torch.zeros(1, dtype=torch.long, device=dev)
    pos_ids = torch.zeros(batch_size, 1, dtype=torch.long, device=dev)
    with torch.no_grad():
        cos, sin = stack.rotary_emb(x, pos_ids)
        for layer in stack.layers:
            layer(x, attention_mask=mask, position_ids=pos_ids, past_key_values=cache, use_cache=True,
                  cache_position=pos, position_embeddings=(cos, sin))
    del cache
    torch.cuda.synchronize(dev)


def _install(stack, mlp_bits, attn_bits) -> int:
    n = 0
    for i, layer in enumerate(stack.layers):
        if isinstance(layer, FusedDecoderLayer):
            continue
        stack.layers[i] = FusedDecoderLayer(layer, i, mlp_bits=mlp_bits, attn_bits=attn_bits)
        n += 1
    return n


def install_fused_backbone(model, *, batch_size: int = 2, max_seq_len: int = 1024, mlp_bits: int | None = None,
                           attn_bits: int = 16) -> int:
    bb = model.backbone_model
    n = _install(bb, mlp_bits, attn_bits)
    _warm(bb, batch_size, max_seq_len)
    return n


def install_fused_depth(model, *, batch_size: int = 2, mlp_bits: int | None = None, attn_bits: int = 16) -> int:
    dm = model.depth_decoder.model
    n = _install(dm, mlp_bits, attn_bits)
    _warm(dm, batch_size, 2 + dm.config.num_codebooks)
    return n
