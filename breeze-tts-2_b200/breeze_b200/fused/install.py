"""Install FusedDecoderLayer on a model's backbone and depth decoder.

Drop-in for models/fused/install.py (install_fused_backbone :16-39,
install_fused_depth :42-65): the same names, keyword arguments and return
value (how many layers were newly wrapped; wrapped layers are left alone).

After wrapping, every fused layer runs decode steps on scratch caches of the
runtime's batch size and cache length (``FusedDecoderLayer.warm_up``, one
position and the longest short prefill). Nothing is tuned -- launch shapes
come from the device -- but the shared per-device workspaces must reach
their final size before the runtime captures its CUDA graphs, because they
may not grow during a capture.
"""

from __future__ import annotations

import torch

from .layer import MAX_NEW_POSITIONS, FusedDecoderLayer


def _wrap_and_warm(decoder, batch_size: int, cache_len: int, mlp_bits, attn_bits) -> int:
    wrapped = 0
    for i, layer in enumerate(decoder.layers):
        if not isinstance(layer, FusedDecoderLayer):
            decoder.layers[i] = FusedDecoderLayer(layer, i, mlp_bits=mlp_bits, attn_bits=attn_bits)
            wrapped += 1
    for layer in decoder.layers:
        for positions in sorted({1, min(MAX_NEW_POSITIONS, cache_len)}):
            layer.warm_up(batch_size, cache_len, positions)
    torch.cuda.synchronize()
    return wrapped


def install_fused_backbone(model, *, batch_size: int = 2, max_seq_len: int = 1024, mlp_bits: int | None = None,
                           attn_bits: int = 16) -> int:
    return _wrap_and_warm(model.backbone_model, batch_size, max_seq_len, mlp_bits, attn_bits)


def install_fused_depth(model, *, batch_size: int = 2, mlp_bits: int | None = None, attn_bits: int = 16) -> int:
    depth = model.depth_decoder.model
    # the depth cache holds the two prefill positions and one per codebook step (reference install.py:52)
    return _wrap_and_warm(depth, batch_size, 2 + depth.config.num_codebooks, mlp_bits, attn_bits)
