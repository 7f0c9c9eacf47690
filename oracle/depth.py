"""One depth-decoder frame restated on the CPU (test oracle only).

Follows DepthDecoderGraph._full_loop (models/cudagraph/depth_decoder_graph.py:
560-660) with the per-layer arithmetic of FusedDecoderLayer.forward
(models/fused/layer.py:87-98): QKV = rms_gemv(x, ln1), attention_step
(oracle/attention.py), O + residual, SiLU(gate) * up = rms_gemv(h, ln2),
down + residual; then the final norm and the fp32 codebook head
(oracle/sampling.py). Every intermediate the GPU keeps in a bf16 buffer is
rounded to bf16 here at the same point. The frame is teacher-forced: each
step's input token is taken from ``tokens`` (the tokens the GPU chose), so a
near-tie decided differently by fp32 summation order cannot derail the
comparison; the oracle returns every step's logits.
"""

from __future__ import annotations

import torch

from . import attention as oa
from . import gemv as og
from . import sampling as osm

EPI_NONE, EPI_SILU_MUL, EPI_ADD_RESIDUAL = 0, 1, 2


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16)


def layer_pass(x, layers, caches, positions, cos, sin, eps):
    """x (R, H) bf16; positions: (row offset, rows, cache position) blocks.
    layers: dicts of dequantized fp32 weights and bf16 norms; caches: list of
    (keys, values) CPU bf16 tensors updated in place."""
    for li, l in enumerate(layers):
        qkv = _bf(og.fused_reference(x, l["wqkv"], l["ln1"], eps, EPI_NONE))
        attn = torch.zeros(x.shape[0], l["wo"].shape[1], dtype=torch.bfloat16)
        keys, values = caches[li]
        for off, n, p in positions:
            out, _, _ = oa.attention_step(qkv[off:off + n], cos[p:p + 1], sin[p:p + 1], p, keys, values,
                                          torch.zeros(n, keys.shape[2]), l["qn"], l["kn"], eps)
            attn[off:off + n] = out
        h = _bf(og.fused_reference(attn, l["wo"], None, eps, EPI_ADD_RESIDUAL, x))
        act = _bf(og.fused_reference(h, l["wgu"], l["ln2"], eps, EPI_SILU_MUL))
        x = _bf(og.fused_reference(act, l["wd"], None, eps, EPI_ADD_RESIDUAL, h))
    return x


def frame_logits(backbone_h, first_tok, tokens, layers, norm_w, head_w, embed, in_proj, cos, sin, n_dec, hkv,
                 head_dim, eps=1e-6):
    """Teacher-forced frame: returns (n_dec, B, vocab) fp32 logits.
    backbone_h (B, E) bf16 (already the audio-embedding width), first_tok (B,),
    tokens (B, n_dec) the sampled tokens of each step."""
    b = backbone_h.shape[0]
    vocab = head_w.shape[2]
    s = 2 + n_dec
    caches = [(torch.zeros(b, hkv, s, head_dim, dtype=torch.bfloat16),
               torch.zeros(b, hkv, s, head_dim, dtype=torch.bfloat16)) for _ in layers]
    rows = embed.shape[0]
    e = torch.cat([backbone_h, embed[first_tok.clamp(0, rows - 1)]], 0)
    x = _bf(og.fused_reference(e, in_proj, None, eps, EPI_NONE))
    x = layer_pass(x, layers, caches, [(0, b, 0), (b, b, 1)], cos, sin, eps)
    out = [osm.head(x[b:2 * b], head_w[0], True, norm_w, eps)]
    for j in range(1, n_dec):
        e = embed[(tokens[:, j - 1] + j * vocab).clamp(0, rows - 1)]
        x = _bf(og.fused_reference(e, in_proj, None, eps, EPI_NONE))
        x = layer_pass(x, layers, caches, [(0, b, j + 1)], cos, sin, eps)
        out.append(osm.head(x, head_w[j], True, norm_w, eps))
    return torch.stack(out, 0)
